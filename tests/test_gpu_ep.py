"""Multi-GPU: expert-parallel forward equals the single-GPU forward bit for
bit (tests/multigpu/ep_check.py under torchrun), through both exchanges
(peer memory and NCCL).  Skipped with fewer than two visible GPUs."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _ngpu():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _run(n, *extra):
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29531",
           os.path.join(ROOT, "tests", "multigpu", "ep_check.py"), *extra]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    return subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)


@pytest.mark.parametrize("extra", [
    ("--transport", "peer", "--graph"),             # BF16: NVLink peer-memory exchange (permute on 32 SMs
                                                    # beside the dense GEMM), eager + CUDA graph
    ("--transport", "peer", "--uneven"),            # one rank with no tokens, the others ragged
    ("--transport", "peer", "--overflow"),          # an over-capacity batch is refused on every rank, then exact
    ("--transport", "peer", "--peer-timeout"),      # a rank that never joins: bounded wait, TIMEOUT, exchange closed
    ("--transport", "peer", "--dispatch", "bulk", "--dispatch-sms", "0", "--graph"),  # bulk-copy permute in line
    ("--transport", "peer", "--dispatch", "bulk", "--dispatch-sms", "16", "--uneven"),  # ... beside the dense GEMM
    ("--transport", "peer", "--dispatch", "threads", "--dispatch-sms", "0"),           # thread permute in line
    ("--transport", "nccl"),                        # the NCCL all-to-all-v exchange
    ("--transport", "nccl", "--uneven"),
    ("--config", "proxy_tiny", "--tokens", "777"),  # F32 layer (NCCL exchange)
    ("--config", "pro", "--tokens", "4000", "--transport", "peer"),        # E = 64, k = 6 over 2/4/8 owners
    ("--config", "max_layer", "--tokens", "2000", "--transport", "peer"),  # E = 128, k = 8
    ("--config", "max_layer", "--tokens", "2000", "--transport", "peer", "--dispatch", "bulk",
     "--dispatch-sms", "16"),
])
def test_expert_parallel_matches_single_gpu(extra):
    n = min(_ngpu(), 8)
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    r = _run(n, *extra)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert '"ok": true' in r.stdout, r.stdout[-3000:]
