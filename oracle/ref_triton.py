"""Builds the reference's own GPU kernels for B200 — TEST INFRASTRUCTURE ONLY.

The reference's hot path is a set of Triton kernels
(python/dli_ops/aot/<op>/kernel.py) that its build compiles ahead of time to
cubins and launches through the CUDA driver with grids fixed in
python/dli_ops/aot/<op>/template.cc. This recipe compiles those kernel
sources, read where they lie in a checkout of the reference, for sm_100a with
the same Triton call the reference's generator makes
(tools/build_triton_aot_ops.py:86-114: an ASTSource with the constexpr and
divisibility hints of one specialisation, num_warps 4, num_stages 3), and
writes into oracle/_ref/triton/:

    <id>.cubin   the compiled kernel
    <id>.json    kernel symbol, shared memory, warps, and its launch
                 parameters (the non-constexpr arguments in order, then the two
                 scratch pointers a Triton 3.6 kernel takes last)

Specialisations: the entries of the reference's AOT table that the benchmark
workloads reach (single linear at K=1024, the CNN's fully-connected layers at
K=4096, its first convolution, decode attention at head_dim 128), plus the
same linear kernel specialised at the Qwen2-7B decode projection widths
(K = 3584, 18944), which the reference's table lacks.

tests/test_ref_triton_gpu.py launches them on the GPU next to this
repository's kernels: parity against the reference's own GPU results and a
timing of both. Nothing in the product path reads oracle/_ref.

    python oracle/ref_triton.py <reference checkout>   (or DLI_REFERENCE_ROOT)
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys
from pathlib import Path

OUT = Path(__file__).resolve().parent / "_ref" / "triton"

# id -> (operator dir, kernel name, signature as the reference's table writes it)
_F, _I = "*fp32", "i32"
SPECS = {
    "linear_k1024_b1": ("linear", "linear_kernel", (_F, _F, _F, _F, _I, _I, "1024", "1", "16", "16", "32")),
    "linear_k4096_b1": ("linear", "linear_kernel", (_F, _F, _F, _F, _I, _I, "4096", "1", "16", "16", "32")),
    "linear_k3584_b0": ("linear", "linear_kernel", (_F, _F, _F, _F, _I, _I, "3584", "0", "16", "16", "32")),
    "linear_k18944_b0": ("linear", "linear_kernel", (_F, _F, _F, _F, _I, _I, "18944", "0", "16", "16", "32")),
    "conv_c3_k3x3_b1": ("conv2d", "conv2d_kernel", (_F, _F, _F, _F) + (_I,) * 11 + ("3", "3", "3", "1", "128")),
    "attention_q1_k512_d128_c1": ("attention", "attention_kernel",
                                  (_F, _F, _F, _F, "1", "512", "128", "1", repr(1 / 128 ** 0.5), "16", "32", "128")),
    "attention_q1_k2048_d128_c1": ("attention", "attention_kernel",
                                   (_F, _F, _F, _F, "1", "2048", "128", "1", repr(1 / 128 ** 0.5), "16", "32", "128")),
    "attention_q128_k128_d128_c1": ("attention", "attention_kernel",
                                    (_F, _F, _F, _F, "128", "128", "128", "1", repr(1 / 128 ** 0.5), "16", "32",
                                     "128")),
}


def _number(text: str):
    for cast in (int, float):
        try:
            return cast(text)
        except ValueError:
            pass
    return None


def _load(reference: Path, op: str):
    path = reference / "python" / "dli_ops" / "aot" / op / "kernel.py"
    spec = importlib.util.spec_from_file_location(f"dli_reference_{op}_kernel", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def compile_one(reference: Path, spec_id: str) -> dict:
    import triton
    from triton.backends.compiler import GPUTarget

    op, name, signature = SPECS[spec_id]
    kernel = getattr(_load(reference, op), name)
    constexprs = {kernel.arg_names[i]: _number(s) for i, s in enumerate(signature) if _number(s) is not None}
    types = {kernel.arg_names[i]: ("constexpr" if kernel.arg_names[i] in constexprs else s)
             for i, s in enumerate(signature)}
    src = triton.compiler.ASTSource(fn=kernel, constexprs=constexprs, signature=types, attrs={})
    compiled = triton.compile(src, target=GPUTarget("cuda", 100, 32), options={"num_warps": 4, "num_stages": 3})
    meta = compiled.metadata
    params = [f"{arg}:{types[arg]}" for arg in kernel.arg_names if types[arg] != "constexpr"]
    params += ["global_scratch:*i8", "profile_scratch:*i8"]
    info = {"id": spec_id, "op": op, "symbol": meta.name, "shared": int(meta.shared), "num_warps": int(meta.num_warps),
            "params": params, "global_scratch_size": int(getattr(meta, "global_scratch_size", 0)),
            "profile_scratch_size": int(getattr(meta, "profile_scratch_size", 0)),
            "constexprs": {k: v for k, v in constexprs.items()}, "triton": triton.__version__}
    OUT.mkdir(parents=True, exist_ok=True)
    (OUT / f"{spec_id}.cubin").write_bytes(compiled.asm["cubin"])
    (OUT / f"{spec_id}.json").write_text(json.dumps(info, indent=1))
    return info


def build(reference: Path) -> list[dict]:
    """Compiles every spec whose cubin is missing or older than its kernel source."""
    done = []
    for spec_id, (op, _, _) in SPECS.items():
        src = reference / "python" / "dli_ops" / "aot" / op / "kernel.py"
        cubin = OUT / f"{spec_id}.cubin"
        if cubin.exists() and (OUT / f"{spec_id}.json").exists() and cubin.stat().st_mtime >= src.stat().st_mtime:
            continue
        done.append(compile_one(reference, spec_id))
    return done


def main() -> int:
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DLI_REFERENCE_ROOT", "")
    if not root or not (Path(root) / "python" / "dli_ops" / "aot").exists():
        print(f"reference checkout not found at {root!r}", file=sys.stderr)
        return 1
    for info in build(Path(root)):
        print(info["id"], info["symbol"], "shared", info["shared"], "params", len(info["params"]))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
