"""Expert parallelism on all the box's GPUs (2, 4 or 8): kc_moe_ffn with each
rank holding a contiguous block of the experts, against one GPU holding all of
them (run with -m gpu; skipped on a box with fewer than 2 GPUs). The ranks run
tests/ep_worker.py under torch.distributed.run; its cases cover both exchange
paths (peer memory up to 32 tokens per rank, NCCL above)."""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
HERE = os.path.dirname(os.path.abspath(__file__))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_expert_parallel_matches_single_gpu():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = max(w for w in (2, 4, 8) if w <= torch.cuda.device_count())
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr=127.0.0.1", f"--master-port={free_port()}", os.path.join(HERE, "ep_worker.py")]
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    lines = [l for l in p.stdout.splitlines() if l.startswith("[")]
    assert lines, p.stdout[-2000:] + p.stderr[-4000:]
    res = json.loads(lines[-1])
    bad = [r for r in res if not r["ok"]]
    assert p.returncode == 0 and not bad, json.dumps(bad)[:2000] + p.stderr[-2000:]
    # The small cases exercise the bit-exact int8 path end to end.
    assert any(r.get("out_bit_exact") for r in res)
