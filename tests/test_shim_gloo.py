"""Host logic of the tensor-parallel all-reduce on CPU: two gloo ranks run the vLLM-side set-up
(NvlinkAllReduce, the port of patches/vllm/gfx906_host_allreduce.py) against a host-only fake
of the operator library that uses the real shared-memory registry of libb2skinny.so for the
rendezvous. Checks the exchange of handles, the unlink, the rank-order sum against gloo's
all_reduce, and that a rank which never joins is reported instead of waited for."""

from __future__ import annotations

import ctypes as C
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


class FakeOps:
    """Host-only stand-in for torch.ops.gfx906_skinny's all-reduce operators. Buffers are faked
    as 64-byte blobs in the real registry; the all-reduce adds all ranks' tensors in rank order
    (gathered through gloo), the contract of the device kernel."""

    def __init__(self, lib, join=True):
        self.lib, self.join, self.reg = lib, join, {}
        self.unlinked = []

    def hostar_max_bytes(self):
        return 128 * 1024

    def _create(self, name, rank, world, create):
        reg = C.c_void_p()
        rc = self.lib.b2_registry_open(name.encode(), world, 1 if create else 0, C.byref(reg))
        if rc:
            raise RuntimeError(self.lib.b2_last_error().decode())
        if self.join:
            blob = (C.c_ubyte * 64)(*([rank + 1] * 64))
            assert self.lib.b2_registry_put(reg, rank, blob) == 0
        h = len(self.reg)
        self.reg[h] = (reg, rank, world)
        return h

    def hostar_create(self, name, slot_bytes, create):
        return self._create(name, 0 if create else 1, 2, create)

    def nvar_create(self, name, slot_bytes, rank, world):
        return self._create(name, rank, world, rank == 0)

    def nvar_connect(self, handle):
        reg, rank, world = self.reg[handle]
        out = (C.c_ubyte * 64)()
        for peer in range(world):
            if self.lib.b2_registry_get(reg, peer, out) != 0:
                raise RuntimeError(f"rank {peer} has not joined the all-reduce yet")
            assert bytes(out) == bytes([peer + 1] * 64)

    def hostar_unlink(self, name):
        self.unlinked.append(name)
        self.lib.b2_registry_unlink(name.encode())

    def _sum(self, t):
        parts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
        dist.all_gather(parts, t)
        acc = torch.zeros_like(t, dtype=torch.float32)
        for p in parts:
            acc = acc + p.float()
        return acc.to(t.dtype)

    def hostar_allreduce(self, t, handle, rank):
        assert rank == self.reg[handle][1]
        return self._sum(t)

    def nvar_allreduce(self, t, handle):
        return self._sum(t)

    def nvar_status(self, handle, clear):
        return 0

    def w4gemm_ar(self, x, w_q, w_zp, w_s, handle):
        """This rank's K-shard GEMM as an fp32 partial, summed over ranks in rank order and
        rounded once (the fused kernel's contract)."""
        from oracle import skinny_oracle as so

        part = so.w4_ref(x.numpy(), w_q.numpy(), w_zp.numpy(), w_s.numpy()).astype("float32")
        return self._sum(torch.from_numpy(part)).half()

    def w4gemm_ar_rmsnorm(self, x, w_q, w_zp, w_s, handle, residual, weight, eps):
        from oracle import skinny_oracle as so

        y = self.w4gemm_ar(x, w_q, w_zp, w_s, handle)
        out, res = so.add_rmsnorm_ref(y.numpy(), residual.numpy(), weight.numpy(), eps)
        residual.copy_(torch.from_numpy(res))
        return torch.from_numpy(out)


def _worker(rank, world, port, scenario, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, str(ROOT))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import __graft_entry__ as entry

        entry.load_package()
        from mi50_vllm_lab_b200 import capi, vllm_shim
        from oracle import skinny_oracle as so

        lib = capi.lib()
        group = dist.new_group(backend="gloo")
        if scenario == "ok":
            fake = FakeOps(lib)
            ar = vllm_shim.NvlinkAllReduce(group, rank, list(range(world)), ops=fake)
            g = torch.Generator().manual_seed(100 + rank)
            for it in range(50):
                dt = torch.float16 if it % 3 else torch.float32
                x = (torch.randn(8 * 64, generator=g) * 10 ** (it % 4 - 1)).to(dt)
                assert ar.should_use(x)
                y = ar.all_reduce(x)
                parts = [torch.empty_like(x) for _ in range(world)]
                dist.all_gather(parts, x)
                want = so.allreduce_ref([p.numpy() for p in parts])
                assert (y.numpy() == want).all() or (y.numpy().view("u1") == want.view("u1")).all()
                if dt == torch.float32 and world == 2:
                    ref = x.clone()
                    dist.all_reduce(ref)  # gloo: a + b, the same single rounding
                    assert torch.equal(y, ref)
            assert not ar.should_use(torch.zeros(3, dtype=torch.float16))        # 6 bytes
            assert not ar.should_use(torch.zeros(8, dtype=torch.int32))          # dtype
            assert not ar.should_use(torch.zeros(1 << 17, dtype=torch.float16))  # > max bytes
            if rank == 0:
                assert len(fake.unlinked) == 1
            # row-parallel layer + residual add + RMSNorm through the shim: every rank passes
            # its K-shard and the same residual; the residual is updated in place, every rank
            # gets the same result, and it matches the unsharded layer's oracle
            M, ks, N, G = 4, 256, 128, 128
            x, qw, qz, sc = so.gen_w4(M, ks * world, N, G, seed=3)
            xs = torch.from_numpy(x[:, rank * ks:(rank + 1) * ks].copy())
            qws = torch.from_numpy(qw[rank * ks // 8:(rank + 1) * ks // 8].copy())
            qzs = torch.from_numpy(qz[rank * ks // G:(rank + 1) * ks // G].copy())
            scs = torch.from_numpy(sc[rank * ks // G:(rank + 1) * ks // G].copy())
            gr = torch.Generator().manual_seed(9)
            res0 = (torch.randn(M, N, generator=gr) * 2).half()
            wn = (1 + torch.rand(N, generator=gr) * 0.2).half()
            res = res0.clone()
            out = ar.w4_gemm_all_reduce_rmsnorm(xs, qws, qzs, scs, res, wn, 1e-6)
            assert not torch.equal(res, res0)  # updated in place
            for t in (out, res):
                parts = [torch.empty_like(t) for _ in range(world)]
                dist.all_gather(parts, t)
                assert all(torch.equal(parts[0], q) for q in parts[1:])
            y_full = so.w4_ref(x, qw, qz, sc).astype("float16")
            ref_out, ref_res = so.add_rmsnorm_ref(y_full, res0.numpy(), wn.numpy(), 1e-6)
            # the sharded fp32 partials and the float64 full GEMM round apart by an ulp at most
            assert so.fp16_ulp_distance(res.numpy(), ref_res).max() <= 1
            assert so.fp16_ulp_distance(out.numpy(), ref_out).max() <= 3
            result_q.put((rank, "ok"))
        else:  # rank 1 never publishes its buffer: rank 0's connect must raise, not hang
            fake = FakeOps(lib, join=(rank == 0))
            try:
                vllm_shim.NvlinkAllReduce(group, rank, list(range(world)), ops=fake)
                result_q.put((rank, "no error"))
            except RuntimeError as e:
                result_q.put((rank, "not joined" if "has not joined" in str(e) else f"other: {e}"))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        result_q.put((rank, f"exception: {type(e).__name__}: {e}"))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(world, scenario):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    out = {}
    while not q.empty():
        r, v = q.get()
        out[r] = v
    return out



@pytest.mark.parametrize("world", [2, 3])
def test_rendezvous_and_rank_order_sum(built, world):
    out = _spawn(world, "ok")
    assert out == {r: "ok" for r in range(world)}, out


def test_rank_that_never_joins_is_reported(built):
    out = _spawn(2, "missing")
    # both ranks connect after the barrier; each sees rank 1's buffer missing
    assert out.get(0) == "not joined" and out.get(1) == "not joined", out
