"""CPU, world_size 2 (gloo): the expert-parallel data flow of one layer
forward -- per-expert count exchange, the library's exchange plan
(noor_moe_ep_plan), all-to-all-v of the token rows, grouped expert compute
on the receiving rank, the reverse all-to-all-v and the rank-order combine --
reproduces the single-process ParallelFFN forward.  Expert math runs in the
oracle; the layout and plan rules are the GPU path's."""
import ctypes
import importlib
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, tokens_per_rank, q):
    try:
        sys.path.insert(0, ROOT)
        import torch
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        pkg = importlib.import_module("noor_-_bangla_ai_b200")
        from oracle import oracle as O
        W = pkg.workloads
        cfg = W.LayerConfig("ep", 64, 32, 8, 2, 32, 64, W.F32, seed=21)
        w = W.make_weights(cfg)
        T = tokens_per_rank[rank]
        x = W.make_tokens(cfg, seed_offset=1 + 7919 * rank, tokens=max(T, 1))[:T]
        E, k, d, G = cfg.n_experts, cfg.top_k, cfg.d_model, world
        El = E // G
        idx, wt, counts = O.route(x, w.gate, w.bias, w.scales, k) if T else (
            np.zeros((0, k), np.int32), np.zeros((0, k), np.float32), np.zeros(E, np.int64))
        # send layout: expert segments in expert order; inside a segment picks in
        # (slot, token) order -- the GPU's order for a single token block
        seg = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
        cursor = seg[:-1].copy()
        dst = np.zeros((T, k), np.int64)
        for slot in range(k):
            for t in range(T):
                e = idx[t, slot]
                dst[t, slot] = cursor[e]
                cursor[e] += 1
        send = np.zeros((int(seg[-1]), d), np.float32)
        for t in range(T):
            for slot in range(k):
                send[dst[t, slot]] = x[t]
        # count exchange: rank r receives every rank's counts for r's experts
        cin = torch.from_numpy(counts.copy())
        cout = torch.zeros(E, dtype=torch.int64)
        dist.all_to_all_single(cout, cin)
        counts_recv = cout.numpy().copy()
        lib = pkg.api.lib()
        lib.noor_moe_ep_plan.argtypes = [ctypes.c_void_p] * 2 + [ctypes.c_int] * 3 + [ctypes.c_void_p] * 7
        sr, so, rr, ro = (np.zeros(G, np.int64) for _ in range(4))
        row, mt, wi = (np.zeros(G * El + 1, np.int32) for _ in range(3))
        P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
        assert lib.noor_moe_ep_plan(P(counts), P(counts_recv), E, G, 128, P(sr), P(so), P(rr), P(ro), P(row),
                                    P(mt), P(wi)) == 0
        recv = torch.zeros((int(rr.sum()), d), dtype=torch.float32)
        dist.all_to_all_single(recv, torch.from_numpy(send), output_split_sizes=rr.tolist(),
                               input_split_sizes=sr.tolist())
        recv = recv.numpy()
        y = np.zeros_like(recv)
        for j in range(G * El):
            a, b = row[j], row[j + 1]
            if b > a:
                e = rank * El + wi[j]
                y[a:b] = O.glu_ffn(recv[a:b], w.w_gate[e], w.w_up[e], w.w_down[e], 1)
        back = torch.zeros((send.shape[0], d), dtype=torch.float32)
        dist.all_to_all_single(back, torch.from_numpy(y), output_split_sizes=sr.tolist(),
                               input_split_sizes=rr.tolist())
        back = back.numpy()
        out = np.zeros((T, d), np.float32)
        if T:
            moe = np.zeros((T, d), np.float32)
            for slot in range(k):
                moe = (moe + wt[:, slot:slot + 1] * back[dst[:, slot]]).astype(np.float32)
            dense = O.glu_ffn(x, w.dense_gate, w.dense_up, w.dense_down, 0)
            out = ((dense + moe) * W.inv_sqrt2()).astype(np.float32)
            ref, ridx, _, _ = O.parallel_forward(w, x, k)
            err = float(np.linalg.norm(out - ref) / np.linalg.norm(ref))
        else:
            err = 0.0
        q.put((rank, err, int(counts_recv.sum()), int(rr.sum())))
        dist.destroy_process_group()
    except Exception as ex:  # pragma: no cover - reported to the parent
        import traceback
        q.put((rank, "error", traceback.format_exc(), 0))


@pytest.mark.parametrize("tokens", [(50, 70), (0, 90)])
def test_ep_two_ranks_gloo(tokens):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, tokens, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert r[1] != "error", r[2]
        assert r[1] <= 1e-6, r
        assert r[2] == r[3]
