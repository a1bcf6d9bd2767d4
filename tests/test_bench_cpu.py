"""The bench line's bookkeeping on the CPU: the algorithmic bytes behind `roofline.achieved`
(the TinyLlama-1.1B-shaped Q4_K_M mix of BASELINE config 3) and the `config` object that both
arms print, so the driver compares like with like."""
import bench


def test_weight_bytes_of_the_tinyllama_mix():
    # Q4_K: 144 B per 256 weights; Q6_K: 210 B per 256 (Q4KTensor.cs / Q6KTensor.cs block sizes)
    c = bench.TINYLLAMA
    H, F, V, L = c["hidden"], c["ffn_hidden"], c["vocab_size"], c["n_layers"]
    kd = c["n_kv_heads"] * c["head_dim"]
    q4 = L * (H * H + kd * H + H * H + 2 * F * H)  # wq, wk, wo, gate, up
    q6 = L * (kd * H + H * F) + V * H               # wv, down, output head
    want = q4 * 144 / 256 + q6 * 210 / 256
    assert bench.weight_bytes_per_token(c) == want == 667152384


def test_step_bytes_add_the_kv_rows_read():
    c = bench.TINYLLAMA
    w = bench.weight_bytes_per_token(c)
    kv_row = 2 * c["n_kv_heads"] * c["head_dim"] * 4  # fp32 K and V of one position, one layer
    for ctx in (1, 2048, 2064):
        extra = bench.step_bytes(c, ctx) - w
        assert extra >= c["n_layers"] * kv_row * ctx
        assert extra <= c["n_layers"] * kv_row * ctx + 64 * 1024  # plus the token's small vectors


def test_both_arms_share_the_config():
    for world in (1, 2, 8):
        cfg = bench.bench_config(world)
        assert cfg["global_batch"] == world and cfg["seq_len"] == bench.PROMPT
        assert cfg["parallelism"].startswith(f"replica x{world}")
        assert "workload" in cfg
