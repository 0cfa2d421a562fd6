"""Generate the residual add + RMSNorm fixtures in this folder by running vLLM's own code.

The reference's models run vLLM's ``fused_add_rms_norm`` on the all-reduced output of o_proj and
down_proj. vLLM is a third-party dependency of the reference (its fork is not vendored in the
reference checkout); the version installed in the build image is 0.22.0. This script calls the
op's reference implementation, ``vllm.ir.ops.layernorm.fused_add_rms_norm`` ("native" provider,
vllm/ir/ops/layernorm.py:40-58), with torch on the CPU, on seeded inputs, and stores inputs and
outputs as .npz:

    python tests/golden/make_golden_rmsnorm.py

The fixtures are committed; nothing at test time imports vLLM.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# name, M, N, eps, y scale, residual scale, weight spread, seed
CASES = [
    ("rmsnorm_m1_n256", 1, 256, 1e-6, 4.0, 1.0, 0.1, 31),
    ("rmsnorm_m2_n5120", 2, 5120, 1e-6, 8.0, 2.0, 0.2, 32),
    ("rmsnorm_m8_n2048", 8, 2048, 1e-5, 1.0, 1.0, 0.5, 33),
    # large values (the sum of squares far above fp16 range; x near the top of fp16), a row
    # of zeros (eps alone sets the scale) and a row of tiny values
    ("rmsnorm_m4_n1024_edges", 4, 1024, 1e-6, 2000.0, 500.0, 1.0, 34),
]


def main() -> None:
    import vllm
    from vllm.ir.ops import layernorm

    impl = layernorm.fused_add_rms_norm.impls["native"].impl_fn
    for name, M, N, eps, ys, rs, wspread, seed in CASES:
        rng = np.random.Generator(np.random.PCG64(seed))
        y = (rng.standard_normal((M, N)) * ys).astype(np.float16)
        res = (rng.standard_normal((M, N)) * rs).astype(np.float16)
        w = (1.0 + rng.uniform(-wspread, wspread, size=N)).astype(np.float16)
        if name.endswith("edges"):
            y[1] = 0
            res[1] = 0
            y[2] = (rng.standard_normal(N) * 1e-3).astype(np.float16)
            res[2] = (rng.standard_normal(N) * 1e-4).astype(np.float16)
        out, new_res = impl(torch.from_numpy(y), torch.from_numpy(res), torch.from_numpy(w), eps)
        np.savez_compressed(HERE / f"{name}.npz", y=y, residual=res, weight=w,
                            eps=np.float64(eps), out=out.numpy(), new_residual=new_res.numpy(),
                            vllm_version=np.str_(vllm.__version__))
        print(f"{name}: M={M} N={N} eps={eps} (vLLM {vllm.__version__})")


if __name__ == "__main__":
    main()
