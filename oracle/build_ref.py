"""Compiles the reference's own GPU kernels for sm_100 into oracle/_ref/ —
TEST INFRASTRUCTURE ONLY (golden-vector generation; never the product path).

Sources, compiled where they lie in the reference tree (read-only, nothing
copied into this repository):
  * research/vadd_emitted.ttir, research/rowsum_emitted.ttir — TTIR written
    by TileTriton's own emitter for the cuTile `vadd` (tile 1024) and
    `rowsum` (tile 64 x 128, TMA descriptors) kernels of test/runtests.jl;
    compiled with the recipe of bench/compile_ttir.py:16-19.
  * research/matmul_emitted.ttir — TileTriton's TTIR for the tf32 `matmul`
    kernel of test/runtests.jl:70-84 (128 x 128 x 32 tiles, 8 warps as that
    test launches it, device-built TMA descriptors).
  * bench/bench_compile.py:45-57 — the Python-Triton twin of the persistent
    column softmax, compiled with TILE = 1024 (the test/runtests.jl:120 case)
    and with TILE = 16384 (the BASELINE 4096 x 16384 config).

The installed triton is 3.6.0; the reference pins 3.7.1 (CondaPkg.toml:8),
which is not installable offline. Outputs: <name>.cubin + <name>.json
(launch metadata). Usage: python oracle/build_ref.py <reference tree>
(or $CTB_REFERENCE_ROOT). Run here (needs the reference tree); the GPU box only
loads the results.
"""
import ast
import json
import os
import sys

# The reference tree: first argument, else $CTB_REFERENCE_ROOT (no default).
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CTB_REFERENCE_ROOT", "")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref")


def _write(name, k):
    with open(os.path.join(OUT, name + ".cubin"), "wb") as f:
        f.write(k.asm["cubin"])
    md = {f: getattr(k.metadata, f)
          for f in ("name", "num_warps", "warp_size", "shared", "global_scratch_size",
                    "global_scratch_align")
          if hasattr(k.metadata, f)}
    with open(os.path.join(OUT, name + ".json"), "w") as f:
        json.dump(md, f)
    return md


def main():
    if not os.path.isdir(REF):
        print("reference tree not present; nothing to build")
        return 0
    from triton.backends.compiler import GPUTarget
    from triton.compiler import ASTSource, compile as tt_compile

    os.makedirs(OUT, exist_ok=True)
    target = GPUTarget("cuda", 100, 32)
    for name in ("vadd", "rowsum"):
        src = os.path.join(REF, "research", f"{name}_emitted.ttir")
        k = tt_compile(src, target=target, options={"num_warps": 4, "num_stages": 3})
        print(name, _write(f"{name}_ttir", k))

    src = os.path.join(REF, "research", "matmul_emitted.ttir")
    k = tt_compile(src, target=target, options={"num_warps": 8, "num_stages": 3})
    print("matmul", _write("matmul_ttir", k))

    # Python-twin softmax: take the function definition from the reference
    # file's syntax tree (the module itself writes files on import).
    path = os.path.join(REF, "bench", "bench_compile.py")
    tree = ast.parse(open(path).read(), path)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "softmax")
    mod = ast.Module(body=[fn], type_ignores=[])
    import triton
    import triton.language as tl

    ns = {"triton": triton, "tl": tl}
    exec(compile(mod, path, "exec"), ns)
    src = ASTSource(fn=ns["softmax"],
                    signature={"out": "*fp32", "inp": "*fp32", "n_rows": "i32", "n_cols": "i32",
                               "stride_o": "i32", "stride_i": "i32", "TILE": "constexpr"},
                    constexprs={"TILE": 1024})
    k = tt_compile(src, target=target, options={"num_warps": 4, "num_stages": 3})
    print("softmax_py", _write("softmax_py", k))
    # The BASELINE config (4096 vectors of 16384): TILE = 16384, one column per
    # tile as the cuTile example runs it; 16 warps keep the tile in registers.
    src = ASTSource(fn=ns["softmax"],
                    signature={"out": "*fp32", "inp": "*fp32", "n_rows": "i32", "n_cols": "i32",
                               "stride_o": "i32", "stride_i": "i32", "TILE": "constexpr"},
                    constexprs={"TILE": 16384})
    k = tt_compile(src, target=target, options={"num_warps": 16, "num_stages": 3})
    print("softmax_py_16384", _write("softmax_py_16384", k))
    return 0


if __name__ == "__main__":
    sys.exit(main())
