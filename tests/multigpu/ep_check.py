"""Expert-parallel parity check, one process per GPU (run under torchrun).

Every rank routes its own seeded batch through the expert-parallel layer
(experts split E/N per rank, NCCL all-to-all-v between ranks).  Rank 0 then
runs the same batches through a single-GPU handle and compares: the layer is
token-wise and each output row is computed the same way whichever tile holds
it, so outputs, picks and counts must be identical bit for bit.  Prints one
JSON line on rank 0 and exits non-zero on a mismatch.
"""
import argparse
import datetime
import importlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)


def main():
    import torch
    import torch.distributed as dist

    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="edge")
    ap.add_argument("--tokens", type=int, default=3000)
    ap.add_argument("--uneven", action="store_true", help="rank r gets tokens * (r + 1) // N tokens (rank 0 may get 0)")
    ap.add_argument("--transport", choices=("auto", "nccl", "peer"), default="auto",
                    help="nccl: force the NCCL exchange; peer: require the peer-memory exchange")
    ap.add_argument("--graph", action="store_true",
                    help="also replay the forward (device mode) as a captured CUDA graph, twice")
    ap.add_argument("--overflow", action="store_true",
                    help="the last rank first sends a batch above the agreed capacity: every rank must "
                         "report the skipped step, then the next step must be exact")
    ap.add_argument("--peer-timeout", action="store_true",
                    help="failure detection: rank 0 runs a forward that the other ranks leave out; its bounded "
                         "device wait (1 s) must end with NOOR_MOE_ERR_TIMEOUT and close the exchange")
    ap.add_argument("--dispatch", choices=("threads", "bulk"), default=None,
                    help="peer exchange: permute rows with thread loads/stores or with bulk copies")
    ap.add_argument("--dispatch-sms", type=int, default=None,
                    help="peer exchange: run the permute on this many SMs beside the dense up projection")
    args = ap.parse_args()
    if args.dispatch:
        os.environ["NOOR_MOE_DISPATCH"] = args.dispatch
    if args.dispatch_sms is not None:
        os.environ["NOOR_MOE_DISPATCH_SMS"] = str(args.dispatch_sms)
    if args.transport == "nccl":
        os.environ["NOOR_MOE_EP_TRANSPORT"] = "nccl"
    if args.peer_timeout:
        os.environ["NOOR_MOE_PEER_TIMEOUT_MS"] = "1000"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    pkg = importlib.import_module("noor_-_bangla_ai_b200")
    W = pkg.workloads
    cfg = W.CONFIGS[args.config]
    w = W.make_weights(cfg)

    def tokens_of(r):
        return (args.tokens * r) // max(1, world - 1) if args.uneven else args.tokens

    def x_of(r):
        n = tokens_of(r)
        return W.make_tokens(cfg, seed_offset=1 + 7919 * r, tokens=max(n, 1))[:n]

    uid = pkg.api.comm_get_id() if rank == 0 else bytes(pkg.api.lib().noor_moe_comm_id_size())
    t = torch.tensor(list(uid), dtype=torch.uint8, device=dev)
    dist.broadcast(t, 0)
    comm = pkg.api.comm_init_rank(bytes(t.cpu().tolist()), world, rank, local)
    h = pkg.api.Handle(cfg.d_model, cfg.n_experts, cfg.top_k, cfg.expert_ff, cfg.dense_ff, dtype=cfg.dtype,
                       device=local, world_size=world, rank=rank, max_tokens=max(tokens_of(rank), 1), comm=comm)
    h.load_weights(w)
    transport = h.ep_transport
    x = x_of(rank)
    xin = W.bf16_bits(x) if cfg.dtype == W.BF16 else x
    if args.peer_timeout:
        outcome, closed = None, None
        if rank == 0:  # the other ranks never enter the step (no kernel of theirs is in flight)
            try:
                h.forward_host(np.ascontiguousarray(xin))
                outcome = "no error"
            except pkg.api.NoorMoEError as e:
                outcome = "timeout" if e.code == 6 else f"code {e.code}"
            try:
                h.forward_host(np.ascontiguousarray(xin))
                closed = False
            except pkg.api.NoorMoEError as e:
                closed = e.code == 5  # NOOR_MOE_ERR_STATE: the exchange stays closed
        dist.barrier()  # rank 0's failed step has ended before any rank frees its buffers
        h.close()
        pkg.api.comm_destroy(comm)
        flags = [None] * world
        dist.all_gather_object(flags, (transport, outcome, closed))
        ok = flags[0][0] == "peer" and flags[0][1] == "timeout" and flags[0][2] is True
        if rank == 0:
            print(json.dumps({"world": world, "peer_timeout": [f[1:] for f in flags], "ok": ok}), flush=True)
        dist.barrier()
        dist.destroy_process_group()
        return 0 if ok else 1
    overflow = None
    if args.overflow:
        # capacity = the largest max_tokens over the ranks, rounded up to 128
        cap = -(-max(max(tokens_of(r), 1) for r in range(world)) // 128) * 128
        big = W.make_tokens(cfg, seed_offset=99, tokens=cap + 1) if rank == world - 1 else x
        bigin = W.bf16_bits(big) if cfg.dtype == W.BF16 else big
        try:
            h.forward_host(np.ascontiguousarray(bigin))
            overflow = "no error"
        except pkg.api.NoorMoEError as e:
            overflow = "invalid" if e.code == 1 else f"code {e.code}"
    out, idx, wt, counts = h.forward_host(np.ascontiguousarray(xin))
    out2, idx2, _, counts2 = h.forward_host(np.ascontiguousarray(xin))  # second call reuses the plan buffers
    same_twice = bool(np.array_equal(out, out2) and np.array_equal(counts, counts2))
    graph_ok = None
    if args.graph:
        n = xin.shape[0]
        tdt = torch.int16 if cfg.dtype == W.BF16 else torch.float32
        xd = torch.from_numpy(np.ascontiguousarray(xin).view(np.int16) if cfg.dtype == W.BF16 else xin).to(dev)
        od = torch.zeros_like(xd)
        cd = torch.zeros(cfg.n_experts, dtype=torch.int64, device=dev)
        cs = torch.cuda.Stream(dev)
        cs.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(cs):
            h.forward_device(xd.data_ptr(), od.data_ptr(), n, cs.cuda_stream, counts_ptr=cd.data_ptr())
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cs):
            h.forward_device(xd.data_ptr(), od.data_ptr(), n, cs.cuda_stream, counts_ptr=cd.data_ptr())
        od.zero_()
        oks = []
        for _ in range(2):
            g.replay()
            torch.cuda.synchronize(dev)
            h.sync()
            got = od.cpu().numpy()
            got = got.view(np.uint16) if cfg.dtype == W.BF16 else got
            oks.append(bool(np.array_equal(got, out) and np.array_equal(cd.cpu().numpy(), counts)))
        del g
        graph_ok = all(oks)
    # one more step from a clean utilization, then the SMEBU update on the
    # device: every rank must hold the global counts and the same new bias
    h.utilization(reset=True)
    h.forward_host(np.ascontiguousarray(xin))
    util_c, util_t = h.utilization()
    h.smebu_update(5.0, 0.9, 0.05)
    bias_ep = h.get_bias()
    h.close()
    pkg.api.comm_destroy(comm)

    # gather every rank's results on rank 0 (CPU objects over the NCCL group)
    gathered = [None] * world
    dist.all_gather_object(gathered, (rank, out, idx, counts))
    ok = True
    flags = [None] * world
    dist.all_gather_object(flags, (transport, overflow, graph_ok, util_c, util_t, bias_ep))
    report = {"world": world, "config": args.config, "tokens": [tokens_of(r) for r in range(world)],
              "same_twice": same_twice, "transport": [f[0] for f in flags]}
    if args.overflow:
        report["overflow"] = [f[1] for f in flags]
    if args.graph:
        report["graph"] = [f[2] for f in flags]
    if rank == 0:
        ref_h = pkg.api.Handle(cfg.d_model, cfg.n_experts, cfg.top_k, cfg.expert_ff, cfg.dense_ff, dtype=cfg.dtype,
                               device=local, max_tokens=max(1, max(tokens_of(r) for r in range(world))))
        ref_h.load_weights(w)
        total_counts = np.zeros(cfg.n_experts, np.int64)
        mismatches = []
        for r, o, i, c in gathered:
            xr = x_of(r)
            if xr.shape[0] == 0:
                continue
            xi = W.bf16_bits(xr) if cfg.dtype == W.BF16 else xr
            ro, ri, _, rc = ref_h.forward_host(np.ascontiguousarray(xi))
            total_counts += rc
            if not np.array_equal(o, ro):
                diff = np.abs(o.astype(np.float64) - ro.astype(np.float64)) if cfg.dtype == W.F32 else None
                mismatches.append({"rank": r, "what": "out", "rows_differ": int((o != ro).any(axis=1).sum())})
            if not np.array_equal(i, ri):
                mismatches.append({"rank": r, "what": "idx"})
        # every rank's counts are the global (all-rank) counts
        for r, o, i, c in gathered:
            if not np.array_equal(c, total_counts):
                mismatches.append({"rank": r, "what": "counts", "got": c.tolist(), "want": total_counts.tolist()})
        # the single-GPU handle recorded every rank's batch once: the global step
        ref_c, ref_t = ref_h.utilization()
        ref_h.smebu_update(5.0, 0.9, 0.05)
        ref_bias = ref_h.get_bias()
        for r, f in enumerate(flags):
            if not (np.array_equal(f[3], ref_c) and f[4] == ref_t):
                mismatches.append({"rank": r, "what": "utilization", "got": [f[3].tolist(), f[4]],
                                   "want": [ref_c.tolist(), ref_t]})
            if not np.array_equal(f[5], ref_bias):
                mismatches.append({"rank": r, "what": "smebu bias"})
        ref_h.close()
        ok = not mismatches and same_twice
        if args.transport == "peer" and any(f[0] != "peer" for f in flags):
            ok = False
        if args.overflow and any(f[1] != "invalid" for f in flags):
            ok = False
        if args.graph and not all(f[2] for f in flags):
            ok = False
        report.update(ok=ok, mismatches=mismatches[:8])
        print(json.dumps(report), flush=True)
    okt = torch.tensor([1 if ok else 0], device=dev)
    dist.broadcast(okt, 0)
    dist.barrier()
    dist.destroy_process_group()
    return 0 if int(okt.item()) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
