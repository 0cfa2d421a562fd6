"""Generate the golden fixtures in this folder by running the reference's OWN reference code.

The reference (0c33/mi50-vllm-lab) ships no stored golden vectors. Its correctness scripts
compute a CPU-runnable reference inline:
  * kernels/check_w4.py:11-18 - float64 dequantization of the Exllama-shuffled layout, and
    kernels/check_w4.py:21 - ``ref = x.double() @ deq``;
  * kernels/bench_skinny.py:44 - ``ref = (x.float() @ w.float().T)``.
This script reads exactly those lines from the reference checkout, executes them with torch on
the CPU (``dev`` bound to the CPU) on seeded inputs, and stores inputs and outputs as .npz. The
scripts themselves cannot be imported (they load vLLM and a GPU library at module level), so only
the reference lines run. Run it in a container that has the reference checkout:

    python tests/golden/make_golden.py /path/to/mi50-vllm-lab

The fixtures are then committed; nothing at test time reads the reference checkout.
"""

from __future__ import annotations

import hashlib
import sys
import textwrap
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
from oracle import skinny_oracle as so  # noqa: E402

# (file, first line, last line) of the reference code that is executed
W4_DEQ_LINES = ("kernels/check_w4.py", 11, 18)
W4_REF_LINES = ("kernels/check_w4.py", 21, 21)
F16_REF_LINES = ("kernels/bench_skinny.py", 44, 44)

W4_CASES = [  # name, M, K, N, G, seed, x_scale (check_w4.py:20 uses randn * 0.5)
    ("w4_g32_m1", 1, 512, 256, 32, 11, 0.5),
    ("w4_g32_m4", 4, 512, 256, 32, 12, 0.5),
    ("w4_g32_m8", 8, 512, 256, 32, 13, 0.5),
    ("w4_g64_m3", 3, 512, 128, 64, 14, 1.0),
    ("w4_g128_m7", 7, 1024, 256, 128, 15, 1.0),
    ("w4_g256_m2", 2, 1024, 160, 256, 16, 1.0),
    ("w4_g128_m5_k2176", 5, 2176, 96, 128, 17, 1.0),
]
F16_CASES = [  # name, M, K, N, seed
    ("f16_m1", 1, 520, 300, 21),
    ("f16_m7", 7, 384, 203, 22),
    ("f16_m8", 8, 640, 136, 23),
    ("f16_m3_k8", 3, 8, 40, 24),
]


def reference_code(root: Path, spec) -> tuple[str, str]:
    fname, lo, hi = spec
    lines = (root / fname).read_text().splitlines()[lo - 1 : hi]
    code = textwrap.dedent("\n".join(lines))
    return code, hashlib.sha256(code.encode()).hexdigest()[:16]


def run_w4(root: Path, x, qw, qz, sc):
    deq_code, h1 = reference_code(root, W4_DEQ_LINES)
    ref_code, h2 = reference_code(root, W4_REF_LINES)
    K = x.shape[1]
    ns = {
        "torch": torch,
        "dev": torch.device("cpu"),
        "K": K,
        "N": qw.shape[1],
        "G": K // sc.shape[0],
        "qw": torch.from_numpy(qw.copy()),
        "qz": torch.from_numpy(qz.copy()),
        "sc": torch.from_numpy(sc.copy()),
        "x": torch.from_numpy(x.copy()),
    }
    exec(deq_code, ns)  # defines u, w, zu, z, deq
    exec(ref_code, ns)  # defines ref
    return ns["ref"].numpy(), h1 + h2


def run_f16(root: Path, x, w):
    code, h = reference_code(root, F16_REF_LINES)
    ns = {"torch": torch, "x": torch.from_numpy(x.copy()), "w": torch.from_numpy(w.copy())}
    exec(code, ns)  # defines ref (float32)
    return ns["ref"].numpy(), h


def main() -> None:
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/mi50-vllm-lab")
    root = Path(sys.argv[1])
    torch.set_num_threads(1)
    for name, M, K, N, G, seed, xs in W4_CASES:
        x, qw, qz, sc = so.gen_w4(M, K, N, G, seed, x_scale=xs)
        ref, h = run_w4(root, x, qw, qz, sc)
        np.savez_compressed(HERE / f"{name}.npz", x=x, qw=qw, qz=qz, sc=sc, ref=ref,
                            ref_code_sha=np.array(h))
        print(name, ref.shape, float(np.abs(ref).max()))
    for name, M, K, N, seed in F16_CASES:
        x, w = so.gen_f16(M, K, N, seed)
        ref, h = run_f16(root, x, w)
        np.savez_compressed(HERE / f"{name}.npz", x=x, w=w, ref=ref, ref_code_sha=np.array(h))
        print(name, ref.shape, float(np.abs(ref).max()))


if __name__ == "__main__":
    main()
