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

CFG = dict(vocab_size=640, hidden=512, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=64, ffn_hidden=1536,
           max_context=96, norm_eps=1e-5, rope_theta=10000.0)
STEPS = 5


def _schemes(O):
    return dict(wq=O.Q4_K, wk=O.Q4_K, wv=O.Q6_K, wo=O.Q4_K, w_gate=O.Q4_K, w_up=O.Q4_K, w_down=O.Q6_K,
                output=O.Q6_K)


def _rank(rank, world, port, out_dir, mega):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), SMALLMIND_MEGA=mega)
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import smallmind_b200 as sm
    from smallmind_b200 import tp
    from oracle import oracle as O
    host = O.make_model(CFG, _schemes(O), seed=17)
    ctx = sm.CudaContext(rank)
    group = tp.TensorParallelGroup(ctx, world, rank)
    model = sm.CudaModel.from_host(ctx, tp.shard_model(host, world, rank))
    group.shard(model)
    kv = sm.KVCache(model, 1, 64)
    prompt = np.random.RandomState(3).randint(0, CFG["vocab_size"], 21).astype(np.int32)
    tok, lg = kv.prefill(0, prompt)
    toks, logits = [tok], [lg]
    for _ in range(STEPS):
        t, l2 = kv.decode([0], [toks[-1]])
        toks.append(int(t[0]))
        logits.append(l2[0])
    np.save(os.path.join(out_dir, f"tok{rank}.npy"), np.array(toks))
    if rank == 0:
        np.save(os.path.join(out_dir, "logits.npy"), np.stack(logits))
        # the unsharded model on this GPU, fed the same tokens
        ref_model = sm.CudaModel.from_host(ctx, host)
        rkv = sm.KVCache(ref_model, 1, 64)
        _, r0 = rkv.prefill(0, prompt)
        ref = [r0]
        for t in toks[:-1]:
            _, r = rkv.decode([0], [t])
            ref.append(r[0])
        np.save(os.path.join(out_dir, "ref.npy"), np.stack(ref))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("mega", ["1", "0"])
def test_tp_decode_matches_single_gpu(tmp_path, world, mega):
    import torch
    import torch.multiprocessing as mp

    from conftest import cosine
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_rank, args=(world, port, str(tmp_path), mega), nprocs=world, join=True)
    logits, ref = np.load(tmp_path / "logits.npy"), np.load(tmp_path / "ref.npy")
    toks = [np.load(tmp_path / f"tok{r}.npy") for r in range(world)]
    for r in range(1, world):
        assert np.array_equal(toks[r], toks[0])
    for step in range(len(ref)):
        assert cosine(logits[step], ref[step]) >= 0.9999, step
        assert int(np.argmax(logits[step])) == int(np.argmax(ref[step])) == int(toks[0][step])
