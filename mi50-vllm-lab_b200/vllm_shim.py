"""The reference's vLLM call sites for this path, ported to the B200 operator library.

The reference patches three vLLM files to route M <= 8 GEMMs and TP all-reduces to its HIP
library. These functions keep those call signatures and return contracts (``None`` = "not
handled, use the stock path") so the patches can point at the B200 library unchanged:

* :func:`w4_skinny`            - ``_gfx906_w4_skinny`` (patches/vllm/exllama.patch:15-32)
* :func:`gptq_gemm_w4`         - ``_gfx906_gptq_gemm_w4_impl`` (patches/vllm/exllama.patch:36-42)
* :func:`gptq_gemm_w4_fake`    - the torch.compile fake impl (patches/vllm/exllama.patch:45-48)
* :func:`skinny8`              - ``_gfx906_skinny8`` (patches/vllm/utils.patch:25-46)
* :class:`NvlinkAllReduce`     - ``Gfx906HostAllReduce`` (patches/vllm/gfx906_host_allreduce.py)

Predicates are wider than the reference's because the sm_100a kernels are: M = 1 is handled
(the reference leaves it to Exllama), N needs only % 32 (W4) or nothing (fp16), K needs % 128
(W4) or % 8 (fp16), and any group size of 32, 64 or a multiple of 128 (the reference gates on
group_size == 32, patches/vllm/exllama.patch:73).
"""

from __future__ import annotations

import os

import torch

from . import ops as _ops


def _valid_group(k: int, groups: int) -> bool:
    if groups <= 0 or k % groups:
        return False
    g = k // groups
    return g in (32, 64) or (g >= 128 and g % 128 == 0)


def w4_skinny(x: torch.Tensor, w_q: torch.Tensor, w_zp: torch.Tensor,
              w_s: torch.Tensor) -> torch.Tensor | None:
    """M = 1..8 4-bit GEMM on the Exllama-shuffled layout, or None when the shape is outside
    the kernel's contract (the caller then runs the stock kernel)."""
    m, k = x.shape
    n = w_q.shape[1]
    if not (1 <= m <= 8 and n % 32 == 0 and k % 128 == 0 and x.dtype == torch.float16
            and _valid_group(k, w_s.shape[0])):
        return None
    return _ops().w4gemm(x.contiguous(), w_q, w_zp, w_s, 0, 0)


def gptq_gemm_w4(x: torch.Tensor, w_q: torch.Tensor, w_zp: torch.Tensor,
                 w_s: torch.Tensor) -> torch.Tensor:
    """Registered behind an opaque custom op so the M-dependent choice happens at run time.
    Shapes the kernel does not take go to vLLM's Exllama kernel when vLLM is importable."""
    out = w4_skinny(x, w_q, w_zp, w_s)
    if out is None:
        from vllm import _custom_ops as vllm_ops  # stock path of the reference (exllama.patch:41)

        out = vllm_ops.gptq_gemm(x, w_q, w_zp, w_s, True, True, 4)
    return out


def gptq_gemm_w4_fake(x: torch.Tensor, w_q: torch.Tensor, w_zp: torch.Tensor,
                      w_s: torch.Tensor) -> torch.Tensor:
    return x.new_empty((x.shape[0], w_q.shape[1]))


def skinny8(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor | None:
    """fp16 GEMM for 1..8 token rows (x [..., K] @ weight[N, K]^T), or None."""
    n = x.numel() // x.size(-1)
    m, k = weight.shape
    if not (1 <= n <= 8 and k % 8 == 0 and x.dtype == torch.float16
            and weight.dtype == torch.float16 and weight.is_contiguous()):
        return None
    x_view = x.reshape(-1, k).contiguous()
    out = _ops().gemm(x_view, weight, 0)
    return out.reshape(*x.shape[:-1], m)


class NvlinkAllReduce:
    """Tensor-parallel all-reduce over NVLink peer memory for one node.

    Same constructor and methods as ``Gfx906HostAllReduce``
    (patches/vllm/gfx906_host_allreduce.py:22-48): rank 0 creates a named rendezvous, the
    others attach after a barrier on the CPU group, rank 0 unlinks the name after a second
    barrier. With two ranks it goes through the reference's own ``hostar_*`` operators; with more
    it uses ``nvar_*``. ``ops`` can be replaced (tests inject a host-only fake).
    """

    _instances = 0

    def __init__(self, cpu_group, rank: int, ranks: list[int], lib: str | None = None,
                 slot_bytes: int | None = None, ops=None):
        import torch.distributed as dist

        if lib:
            torch.ops.load_library(lib)
            ops = ops or torch.ops.gfx906_skinny
        self.ops = ops or _ops()
        self.rank = rank
        self.world = len(ranks)
        self.max_bytes = int(slot_bytes or self.ops.hostar_max_bytes())
        NvlinkAllReduce._instances += 1
        name = [f"/b2_nvar_{os.getpid()}_{ranks[0]}_{NvlinkAllReduce._instances}"
                if rank == 0 else None]
        dist.broadcast_object_list(name, src=ranks[0], group=cpu_group)
        two = self.world == 2
        if rank == 0:
            self.handle = (self.ops.hostar_create(name[0], self.max_bytes, True) if two else
                           self.ops.nvar_create(name[0], self.max_bytes, 0, self.world))
        dist.barrier(group=cpu_group)
        if rank != 0:
            self.handle = (self.ops.hostar_create(name[0], self.max_bytes, False) if two else
                           self.ops.nvar_create(name[0], self.max_bytes, rank, self.world))
        dist.barrier(group=cpu_group)
        self.ops.nvar_connect(self.handle)
        dist.barrier(group=cpu_group)
        if rank == 0:
            self.ops.hostar_unlink(name[0])

    def should_use(self, t: torch.Tensor) -> bool:
        if t.dtype not in (torch.float16, torch.float32) or not t.is_contiguous():
            return False
        nbytes = t.numel() * t.element_size()
        return 0 < nbytes <= self.max_bytes and nbytes % 16 == 0

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.world == 2:
            return self.ops.hostar_allreduce(t, self.handle, self.rank)
        return self.ops.nvar_allreduce(t, self.handle)

    def w4_gemm_all_reduce(self, x, w_q, w_zp, w_s) -> torch.Tensor:
        """Row-parallel W4 layer: this rank's K-shard GEMM with the all-reduce fused in."""
        return self.ops.w4gemm_ar(x, w_q, w_zp, w_s, self.handle)

    def w4_gemm_all_reduce_rmsnorm(self, x, w_q, w_zp, w_s, residual, weight,
                                   eps: float) -> torch.Tensor:
        """The same layer followed, in the same call, by the decoder layer's residual add +
        RMSNorm (vLLM's fused_add_rms_norm): ``residual`` is updated in place, the normalised
        rows are returned."""
        return self.ops.w4gemm_ar_rmsnorm(x, w_q, w_zp, w_s, self.handle, residual, weight, eps)

    def w4_gemm_all_reduce_packed(self, x, packed, n: int, group_size: int) -> torch.Tensor:
        """w4_gemm_all_reduce on weights repacked at load time (w4_repack); n = output width."""
        return self.ops.w4gemm_ar_packed(x, packed, n, group_size, self.handle)

    def w4_gemm_all_reduce_rmsnorm_packed(self, x, packed, n: int, group_size: int, residual,
                                          weight, eps: float) -> torch.Tensor:
        return self.ops.w4gemm_ar_rmsnorm_packed(x, packed, n, group_size, self.handle, residual,
                                                 weight, eps)

    def status(self, clear: bool = False) -> int:
        return int(self.ops.nvar_status(self.handle, clear))


def enabled_library() -> str:
    """The library path the patched vLLM reads (VLLM_GFX906_SKINNY8_LIB); this package's."""
    from . import lib_path

    return os.environ.get("VLLM_GFX906_SKINNY8_LIB", lib_path())
