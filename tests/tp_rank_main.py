"""One rank of the tensor-parallel GPU test (launched by tests/test_gpu_tp.py through
torch.distributed.run, one process per GPU): builds this rank's shard, decodes,
and rank 0 also runs the unsharded model; results go to numpy files in argv[1]."""
import faulthandler
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

CFG = dict(vocab_size=640, hidden=512, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=64, ffn_hidden=1536,
           max_context=96, norm_eps=1e-5, rope_theta=10000.0)
STEPS = 5


def main(out_dir):
    faulthandler.dump_traceback_later(int(os.environ.get("TP_RANK_STACK_AFTER", "200")), exit=True)  # a stuck rank prints where it is and ends
    import torch
    import torch.distributed as dist
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    import smallmind_b200 as sm
    from smallmind_b200 import tp
    from oracle import oracle as O
    schemes = dict(wq=O.Q4_K, wk=O.Q4_K, wv=O.Q6_K, wo=O.Q4_K, w_gate=O.Q4_K, w_up=O.Q4_K, w_down=O.Q6_K,
                   output=O.Q6_K)
    host = O.make_model(CFG, schemes, seed=17)
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
        ref_model = sm.CudaModel.from_host(ctx, host)
        rkv = sm.KVCache(ref_model, 1, 64)
        _, r0 = rkv.prefill(0, prompt)
        ref = [r0]
        for t in toks[:-1]:
            _, r = rkv.decode([0], [t])
            ref.append(r[0])
        np.save(os.path.join(out_dir, "ref.npy"), np.stack(ref))
    # release the library's objects on every rank while all ranks are alive (the
    # context owns the NCCL communicator), then leave without interpreter teardown:
    # a rank must not sit in CUDA / NCCL clean-up waiting for a peer that has gone
    kv.close()
    model.close()
    if rank == 0:
        rkv.close()
        ref_model.close()
    dist.barrier()
    ctx.close()
    dist.barrier()
    dist.destroy_process_group()
    faulthandler.cancel_dump_traceback_later()
    sys.stdout.flush()
    sys.stderr.flush()
    os._exit(0)


if __name__ == "__main__":
    main(sys.argv[1])
