"""GPU, 2 or 4 processes x 1 GPU each (NCCL): the sequence-sharded module
against the fp32 oracle, outputs and all gradients.  Skipped when fewer GPUs
are visible (the driver's single-GPU test run)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, cases, q_out):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    import elastic_sparse_attention_b200 as esa
    from oracle import compare, naive, pattern
    errs = []
    for (layer, S, Hq, Hkv, D, w, dtype) in cases:
        L = S * world
        g = torch.Generator().manual_seed(layer + 11)
        q, k, v, do = (torch.randn(1, L, h, D, generator=g).to(dev, dtype) for h in (Hq, Hkv, Hkv, Hq))
        sl = slice(rank * S, (rank + 1) * S)
        qs, ks, vs = (t[:, sl].clone().requires_grad_(True) for t in (q, k, v))
        m = esa.SequenceShardedElasticSparseAttention(layer, 8, Hq, D, w, L, num_key_value_heads=Hkv)
        out = m(qs, ks, vs)
        out.backward(do[:, sl].reshape(1, S, Hq * D))
        got = []
        for t in (out.detach(), qs.grad, ks.grad, vs.grad):
            lst = [torch.zeros_like(t) for _ in range(world)]
            dist.all_gather(lst, t.contiguous())
            got.append(torch.cat(lst, dim=1).float())
        if rank == 0:
            idx, mask, _ = pattern.prepared_indices(Hq, w, layer, 8, L, L, L)
            ro, rdq, rdk, rdv = naive.naive_forward_backward_manual(
                q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), do.transpose(1, 2),
                torch.from_numpy(idx).to(dev), torch.from_numpy(mask).to(dev), D ** -0.5, Hq // Hkv)
            want = [ro.transpose(1, 2).reshape(1, L, Hq * D), rdq.transpose(1, 2),
                    rdk.transpose(1, 2), rdv.transpose(1, 2)]
            for a, b in zip(got, want):
                errs.append(compare.within(a.to(dtype), b, dtype))
    if rank == 0:
        q_out.put(errs)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sequence_sharded_gpus(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    cases = [(7, 1024, 8, 2, 128, 64, torch.bfloat16), (3, 768, 4, 4, 128, 64, torch.bfloat16),
             (0, 1024, 8, 2, 128, 64, torch.bfloat16), (5, 512, 4, 2, 64, 64, torch.float16)]
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cases, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    errs = q_out.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    names = [f"{c[0]}/{c[-1]} {t}" for c in cases for t in ("out", "dq", "dk", "dv")]
    bad = [(n, mx, mean) for n, (ok, mx, mean) in zip(names, errs) if not ok]
    assert not bad, bad


class _CudaKernelsOnCpuTensors:
    """The kernel ops the sharded module calls, run by the CUDA library on
    cuda:0 for CPU tensors (copies in and out), so that gloo ranks on one GPU
    exercise the sharded module's exchange and reduction with the real
    kernels."""

    @staticmethod
    def _esa():
        import elastic_sparse_attention_b200 as esa
        return esa

    @classmethod
    def pattern_indices(cls, num_heads, spec, n_rows, device, rows=None, row_offset=0,
                        clamp_len=0):
        esa = cls._esa()
        idx, mask = esa.ops.pattern_indices(num_heads, spec, n_rows, torch.device(DEV_ONE),
                                            rows=None if rows is None else rows.to(DEV_ONE),
                                            row_offset=row_offset, clamp_len=clamp_len)
        return idx.to(device), mask.to(device)

    @classmethod
    def forward(cls, q, k, v, spec, scale, rows=None, row_offset=0, kv_len=None, kv_offset=0,
                out=None):
        esa = cls._esa()
        qd, kd, vd = (t.contiguous().to(DEV_ONE) for t in (q, k, v))
        o, lse = esa.ops.forward(qd, kd, vd, spec, scale, row_offset=row_offset, kv_len=kv_len,
                                 kv_offset=kv_offset)
        o = o.cpu()
        if out is not None:
            out.copy_(o)
            o = out
        return o, lse.cpu()

    @classmethod
    def key_plan(cls, q, k, spec, row_offset=0, kv_len=None, kv_offset=0):
        esa = cls._esa()
        return esa.ops.key_plan(q.contiguous().to(DEV_ONE), k.contiguous().to(DEV_ONE), spec,
                                row_offset=row_offset, kv_len=kv_len, kv_offset=kv_offset)

    @classmethod
    def backward(cls, q, k, v, o, lse, dout, spec, scale, rows=None, row_offset=0, kv_len=None,
                 kv_offset=0, dq=None, dk=None, dv=None, dkv_fp32=False, key_plan=None):
        esa = cls._esa()
        qd, kd, vd, od, dod = (t.contiguous().to(DEV_ONE) for t in (q, k, v, o, dout))
        res = esa.ops.backward(qd, kd, vd, od, lse.to(DEV_ONE), dod, spec, scale,
                               row_offset=row_offset, kv_len=kv_len, kv_offset=kv_offset,
                               dkv_fp32=dkv_fp32, key_plan=key_plan)
        out = []
        for got, buf in zip(res, (dq, dk, dv)):
            got = got.cpu()
            if buf is not None:
                buf.copy_(got)
                got = buf
            out.append(got)
        return tuple(out)


DEV_ONE = "cuda:0"


def _gloo_worker(rank, world, port, case, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import elastic_sparse_attention_b200 as esa
    from oracle import compare, naive, pattern
    layer, S, Hq, Hkv, D, w, dtype = case
    L = S * world
    g = torch.Generator().manual_seed(layer + 11)
    q, k, v, do = (torch.randn(1, L, h, D, generator=g).to(dtype) for h in (Hq, Hkv, Hkv, Hq))
    sl = slice(rank * S, (rank + 1) * S)
    qs, ks, vs = (t[:, sl].clone().requires_grad_(True) for t in (q, k, v))
    m = esa.SequenceShardedElasticSparseAttention(layer, 8, Hq, D, w, L, num_key_value_heads=Hkv,
                                                  ops=_CudaKernelsOnCpuTensors)
    out = m(qs, ks, vs)
    out.backward(do[:, sl].reshape(1, S, Hq * D))
    got = []
    for t in (out.detach(), qs.grad, ks.grad, vs.grad):
        lst = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(lst, t.contiguous())
        got.append(torch.cat(lst, dim=1).float())
    if rank == 0:
        dev = torch.device(DEV_ONE)
        idx, mask, _ = pattern.prepared_indices(Hq, w, layer, 8, L, L, L)
        ro, rdq, rdk, rdv = naive.naive_forward_backward_manual(
            q.transpose(1, 2).to(dev), k.transpose(1, 2).to(dev), v.transpose(1, 2).to(dev),
            do.transpose(1, 2).to(dev), torch.from_numpy(idx).to(dev),
            torch.from_numpy(mask).to(dev), D ** -0.5, Hq // Hkv)
        want = [ro.transpose(1, 2).reshape(1, L, Hq * D), rdq.transpose(1, 2),
                rdk.transpose(1, 2), rdv.transpose(1, 2)]
        q_out.put([compare.within(a.to(dev).to(dtype), b, dtype) for a, b in zip(got, want)])
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,case", [
    (2, (7, 1024, 8, 2, 128, 64, torch.bfloat16)), (2, (3, 768, 4, 4, 128, 64, torch.bfloat16)),
    (2, (0, 1024, 8, 2, 128, 64, torch.bfloat16)), (2, (5, 512, 4, 2, 64, 64, torch.float16)),
    (3, (6, 512, 8, 2, 128, 64, torch.bfloat16))])
def test_sequence_sharded_gloo_ranks_on_one_gpu(world, case):
    """The sequence-sharded module with gloo ranks on the CPU whose kernels run
    on one GPU (each rank's calls are independent launches): the exchange plan,
    the K/V fetch, the reverse dK/dV exchange and the fp32 reduction, with the
    CUDA kernels at their row / kv offsets, against the fp32 oracle."""
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, case, q_out))
             for r in range(world)]
    for p in procs:
        p.start()
    errs = q_out.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    bad = [(t, mx, mean) for t, (ok, mx, mean) in zip(("out", "dq", "dk", "dv"), errs) if not ok]
    assert not bad, (case, bad)


def _one_rank_worker(port, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=0, world_size=1)
    import elastic_sparse_attention_b200 as esa
    g = torch.Generator().manual_seed(9)
    B, L, Hq, Hkv, D, dt = 1, 3000, 8, 2, 128, torch.bfloat16
    q, k, v = (torch.randn(B, L, h, D, generator=g).to(DEV_ONE, dt) for h in (Hq, Hkv, Hkv))
    do = torch.randn(B, L, Hq * D, generator=g).to(DEV_ONE, dt)
    res = []
    for mk in (lambda: esa.SequenceShardedElasticSparseAttention(5, 8, Hq, D, 64, L,
                                                                 num_key_value_heads=Hkv),
               lambda: esa.ElasticSparseAttention(5, 8, Hq, D, 64, L, num_key_value_heads=Hkv)):
        m = mk()
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        if isinstance(m, esa.ElasticSparseAttention):
            out, _ = m(qq.transpose(1, 2), kk.transpose(1, 2), vv.transpose(1, 2))
        else:
            out = m(qq, kk, vv)
        out.backward(do)
        res.append([out.detach(), qq.grad, kk.grad, vv.grad])
    q_out.put([bool(torch.equal(a, b)) for a, b in zip(*res)])
    dist.destroy_process_group()


def test_sequence_sharded_one_rank_is_the_module():
    """A sequence group of one rank runs the one-GPU path: outputs and
    gradients equal those of ElasticSparseAttention on the same tensors."""
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    p = ctx.Process(target=_one_rank_worker, args=(_port(), q_out))
    p.start()
    same = q_out.get(timeout=300)
    p.join(timeout=60)
    assert p.exitcode == 0
    assert all(same), same
