"""Tensor-parallel decode on 2, 4 or 8 GPUs against the single-GPU model.

Each rank (its own process and GPU) builds its shard of the same host model
(smallmind_b200.tp.shard_model), joins the NCCL group and runs a prompt plus
greedy decode steps; rank 0 compares every step's logits with the unsharded
model on one GPU: cosine >= 0.9999 and the same greedy token, and all ranks must
produce the same tokens.  Skipped when the box has fewer GPUs than ranks.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("mega", ["1", "0"])
def test_tp_decode_matches_single_gpu(tmp_path, world, mega):
    """Ranks run tests/tp_rank_main.py under torch.distributed.run (bounded: 300 s)."""
    import subprocess
    import sys

    import torch

    from conftest import cosine
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    env = dict(os.environ, SMALLMIND_MEGA=mega)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", f"--master-port={port}", os.path.join(HERE, "tp_rank_main.py"),
           str(tmp_path)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, (r.stdout[-3000:], r.stderr[-3000:])
    logits, ref = np.load(tmp_path / "logits.npy"), np.load(tmp_path / "ref.npy")
    toks = [np.load(tmp_path / f"tok{r_}.npy") for r_ in range(world)]
    for r_ in range(1, world):
        assert np.array_equal(toks[r_], toks[0])
    for step in range(len(ref)):
        assert cosine(logits[step], ref[step]) >= 0.9999, step
        assert int(np.argmax(logits[step])) == int(np.argmax(ref[step])) == int(toks[0][step])
