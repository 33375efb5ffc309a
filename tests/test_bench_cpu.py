"""The bench's algorithmic byte and FLOP counts (the roofline numerators),
checked against counts made independently here from the cache and weight
layouts: MLX affine group quantization stores, per row of `dim` elements,
dim * bits / 8 bytes of packed codes plus one scale and one bias of two
bytes per group (src/mlx/ops.ts:615-637)."""
import numpy as np

import bench


def test_kv_row_bytes_config5():
    # kv4, head_dim 128, group 64: 64 B of codes + 2 scales + 2 biases, K and V
    assert bench.kv_row_bytes(bench.CFG5) == 2 * (64 + 2 * 2 + 2 * 2) == 144


def test_config5_lengths_and_step_bytes():
    lens = bench.config5_lens()
    assert lens.shape == (64,)
    assert lens.min() >= 1024 and lens.max() <= 32768
    assert int(lens.sum()) == 1_050_397
    keys = 1_050_397 * 8 * 144                 # every key row of every kv head
    q_out = 64 * 32 * 128 * 2 * 2              # fp16 queries in, outputs back
    assert bench.config5_rank_bytes(lens, 8) == keys + q_out == 1_211_105_920


def test_config5_shards_add_up():
    """kv-head shards on N ranks: the per-rank bytes times N is the one-GPU
    total, so the aggregate GB/s of every N counts the same bytes."""
    lens = bench.config5_lens()
    total = bench.config5_rank_bytes(lens, 8)
    for n in (1, 2, 4, 8):
        assert bench.config5_rank_bytes(lens, 8 // n) * n == total


def test_projection_bytes_gemma4_12b_sliding_layer():
    c = bench.CFGP
    rows_w = (16 + 8 + 8) * 256                # Q, K and V output features
    codes = rows_w * 3840 // 2                 # 4-bit weights
    scales_biases = rows_w * (3840 // 64) * 2 * 2
    x_row = 3840 * 2
    q_row = 16 * 256 * 2
    cache_rows = 2 * 8 * (256 // 2 + 2 * (256 // 64) * 2)   # K and V, kv4 group 64
    assert bench.projection_out_features(c) == rows_w
    assert bench.projection_bytes(c, 1) == codes + scales_biases + x_row + q_row + cache_rows \
        == 17_712_896


def test_prefill_flops():
    # config 4: QK^T and PV over 16,384 prior keys plus the causal chunk
    c = bench.CFG4
    want = 0
    for i in range(c["L"]):                    # query row i sees N_prior + i + 1 keys
        want += 2 * 2 * c["Hq"] * c["D"] * (c["N_prior"] + i + 1)
    assert bench.prefill_flops(c) == want
    # the projection prefill chunk: one multiply-add per weight element and token
    assert 2 * 512 * 3840 * bench.projection_out_features(bench.CFGP) == 32_212_254_720


def test_lengths_are_seeded():
    assert np.array_equal(bench.config5_lens(), bench.config5_lens())
