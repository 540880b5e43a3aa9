"""CPU, multi-process (gloo): the sequence-sharded module's exchange plan, KV
fetch, reverse dK/dV exchange and fp32 reduction, with the kernels replaced
by the oracle (the CUDA kernels are checked on their own by the GPU tests).
Each rank runs on its shard; rank 0 compares the gathered output and
gradients with one unsharded oracle run."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import naive, pattern


class OracleOps:
    """The subset of the kernel ops the sharded module calls, computed by the
    fp32 oracle on the CPU (test infrastructure only)."""

    @staticmethod
    def pattern_indices(num_heads, spec, n_rows, device, rows=None, row_offset=0, clamp_len=0):
        pos = rows.cpu().numpy() if rows is not None else np.arange(row_offset, row_offset + n_rows)
        idx, mask = pattern.elastic_indices(pos, num_heads, spec.attention_length, spec.layer_idx,
                                            spec.num_hidden_layers)
        return torch.from_numpy(idx).to(device), torch.from_numpy(mask).to(device)

    @staticmethod
    def _local(q, k, spec, row_offset, kv_len, kv_offset):
        Hq, n = q.shape[1], q.shape[2]
        pos = np.arange(row_offset, row_offset + n)
        # the call's heads are heads [head_offset, head_offset + Hq) of the pattern
        H = spec.pattern_heads or Hq
        idx, mask = pattern.elastic_indices(pos, H, spec.attention_length, spec.layer_idx,
                                            spec.num_hidden_layers)
        idx = idx[spec.head_offset:spec.head_offset + Hq]
        mask = mask[spec.head_offset:spec.head_offset + Hq]
        idx = np.clip(idx, 0, kv_len - 1) - kv_offset
        assert (idx[mask.astype(bool)] >= 0).all() and (idx < k.shape[2]).all()
        return torch.from_numpy(np.clip(idx, 0, None)), torch.from_numpy(mask)

    @classmethod
    def forward(cls, q, k, v, spec, scale, rows=None, row_offset=0, kv_len=None, kv_offset=0,
                out=None):
        idx, mask = cls._local(q, k, spec, row_offset, kv_len, kv_offset)
        do = torch.zeros_like(q)
        o, *_ = naive.naive_forward_backward_manual(q, k, v, do, idx, mask, scale,
                                                    q.shape[1] // k.shape[1])
        o = o.to(q.dtype)
        if out is not None:
            out.copy_(o)
            o = out
        return o, torch.zeros(q.shape[:3])

    @classmethod
    def backward(cls, q, k, v, o, lse, dout, spec, scale, rows=None, row_offset=0, kv_len=None,
                 kv_offset=0, dq=None, dk=None, dv=None, dkv_fp32=False):
        idx, mask = cls._local(q, k, spec, row_offset, kv_len, kv_offset)
        _, gq, gk, gv = naive.naive_forward_backward_manual(q, k, v, dout, idx, mask, scale,
                                                            q.shape[1] // k.shape[1])
        res = []
        for got, buf, ref in ((gq, dq, q), (gk, dk, k), (gv, dv, v)):
            got = got.to(ref.dtype)
            if buf is not None:
                buf.copy_(got)
                got = buf
            res.append(got)
        return tuple(res)


def _worker(rank, world, port, layer, S, Hq, Hkv, D, w, result_q, group_ranks=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import elastic_sparse_attention_b200 as esa
    # the sequence group: all ranks, or a sub-group (every rank takes part in
    # creating it; ranks outside it do no attention work)
    group = dist.new_group(group_ranks) if group_ranks is not None else None
    members = group_ranks if group_ranks is not None else list(range(world))
    if rank not in members:
        dist.barrier()
        dist.destroy_process_group()
        return
    grank, gworld = dist.get_rank(group), dist.get_world_size(group)
    L = S * gworld
    g = torch.Generator().manual_seed(3)
    q, k, v, do = (torch.randn(1, L, h, D, generator=g) for h in (Hq, Hkv, Hkv, Hq))
    sl = slice(grank * S, (grank + 1) * S)
    qs, ks, vs = (t[:, sl].clone().requires_grad_(True) for t in (q, k, v))
    m = esa.SequenceShardedElasticSparseAttention(layer, 8, Hq, D, w, L, num_key_value_heads=Hkv,
                                                  group=group, ops=OracleOps)
    out = m(qs, ks, vs)
    out.backward(do[:, sl].reshape(1, S, Hq * D))
    parts = [out.detach(), qs.grad, ks.grad, vs.grad]
    gathered = []
    for t in parts:
        lst = [torch.zeros_like(t) for _ in range(gworld)]
        dist.all_gather(lst, t.contiguous(), group=group)
        gathered.append(torch.cat(lst, dim=1))
    if grank == 0:
        idx, mask, _ = pattern.prepared_indices(Hq, w, layer, 8, L, L, L)
        ro, rdq, rdk, rdv = naive.naive_forward_backward_manual(
            q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), do.transpose(1, 2),
            torch.from_numpy(idx), torch.from_numpy(mask), D ** -0.5, Hq // Hkv)
        want = [ro.transpose(1, 2).reshape(1, L, Hq * D), rdq.transpose(1, 2),
                rdk.transpose(1, 2), rdv.transpose(1, 2)]
        errs = [float((a - b).abs().max()) for a, b in zip(gathered, want)]
        result_q.put(errs)
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("world,layer,S,Hq,Hkv,D,w,group_ranks",
                         [(2, 7, 96, 4, 2, 16, 16, None),
                          (3, 4, 80, 2, 2, 16, 32, None),
                          (2, 0, 70, 2, 1, 8, 16, None),
                          (2, 5, 64, 8, 4, 16, 16, None),
                          # a sequence group that is not WORLD: peers are
                          # addressed by their rank inside the group
                          (3, 6, 64, 4, 2, 16, 16, [2, 1]),
                          (4, 3, 64, 2, 1, 16, 16, [1, 3])])
def test_sequence_sharded_matches_unsharded(world, layer, S, Hq, Hkv, D, w, group_ranks):
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker,
                         args=(r, world, port, layer, S, Hq, Hkv, D, w, result_q, group_ranks))
             for r in range(world)]
    for p in procs:
        p.start()
    errs = result_q.get(timeout=240)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert max(errs) < 1e-4, errs
