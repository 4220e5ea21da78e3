"""Tensor parallelism and the multi-chunk history window on B200s (BASELINE configs[4] at test
size).  Tolerances as the single-GPU engine tests: latent and history rel-L2 <= 3e-2 against
the fp32 CPU oracle; a tensor-parallel run against the same model on one GPU differs only by
the bf16 all-reduce of the row-parallel partial sums (<= 1e-2)."""
import json
import os
import subprocess
import sys

import pytest
import torch

from fastworld_b200.config import SMALL_TP

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
TOL = 3e-2


def test_history_window_two_chunks_one_gpu():
    """hist_chunks = 2 on one GPU: chunks 0-3 (no history, 1 slot, 2 slots, wrap) vs the oracle."""
    from test_engine_gpu import rollout_vs_oracle
    errs = rollout_vs_oracle(SMALL_TP, 4)
    for e in errs:
        assert all(v < TOL for v in e.values()), e


@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel(world):
    """world 2: the one-shot peer reduction; world 4: the two-shot one (1 head per rank)."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={29533 + world}",
           os.path.join(HERE, "mgpu_tp.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    line = [x for x in r.stdout.splitlines() if x.startswith("TP_RESULT ")]
    assert line, r.stdout[-2000:]
    res = json.loads(line[0][len("TP_RESULT "):])
    print(res)
    assert res["ranks_identical"]
    assert all(s[0] == 0 for s in res["status"])
    assert max(res["oracle_rel"]) < TOL and res["hist_rel"] < TOL
    assert max(res["tp1_rel"]) < 1e-2
    assert res["graph_vs_eager"] < 1e-2
    assert res["nccl_rel"] < 1e-2
