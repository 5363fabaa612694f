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
    args = ap.parse_args()
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
    x = x_of(rank)
    xin = W.bf16_bits(x) if cfg.dtype == W.BF16 else x
    out, idx, wt, counts = h.forward_host(np.ascontiguousarray(xin))
    out2, idx2, _, counts2 = h.forward_host(np.ascontiguousarray(xin))  # second call reuses the plan buffers
    same_twice = bool(np.array_equal(out, out2) and np.array_equal(counts, counts2))
    h.close()
    pkg.api.comm_destroy(comm)

    # gather every rank's results on rank 0 (CPU objects over the NCCL group)
    gathered = [None] * world
    dist.all_gather_object(gathered, (rank, out, idx, counts))
    ok = True
    report = {"world": world, "config": args.config, "tokens": [tokens_of(r) for r in range(world)],
              "same_twice": same_twice}
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
        ref_h.close()
        ok = not mismatches and same_twice
        report.update(ok=ok, mismatches=mismatches[:8])
        print(json.dumps(report), flush=True)
    okt = torch.tensor([1 if ok else 0], device=dev)
    dist.broadcast(okt, 0)
    dist.barrier()
    dist.destroy_process_group()
    return 0 if int(okt.item()) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
