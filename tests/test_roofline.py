"""The algorithmic work counts behind bench.py's roofline fractions (vsa_lm_b200/roofline.py).

Each count is checked against a brute-force restatement of the reference's chunk loop
(vsa_lm/config/bolt3.py:194-276): which chunks consolidate, which keys every token attends to,
when the bank and M_res exist. The headline totals are pinned, so that a change of a formula
shows up as a changed number here and not silently in the bench line.
"""
import pytest

from vsa_lm_b200 import kernels as K
from vsa_lm_b200 import roofline as R
from vsa_lm_b200.workloads import layer_cfg

C = S = 128
SINKS = 4


def _chunk_loop(T: int):
    """The reference forward's chunk loop (bolt3.py:210-272), reduced to its control flow: yields
    (chunk start, chunk length, previous chunk present, bank present) for each chunk and counts
    the consolidations (a full chunk that is not the last one consolidates the previous chunk)."""
    out, n_cons, prev, bank = [], 0, False, False
    for s in range(0, T, C):
        e = min(s + C, T)
        out.append((s, e - s, prev, bank))
        if e - s == C and e < T:
            if prev:
                n_cons += 1
                bank = True
            prev = True
    return out, n_cons


@pytest.mark.parametrize("T", list(range(1, 700)) + [4096, 8191, 8192, 8193, 131072])
def test_consolidation_count_follows_the_reference_loop(T):
    _, n = _chunk_loop(T)
    assert R.n_consolidations(T) == n == K.n_consolidations(T)


@pytest.mark.parametrize("T", [1, 5, 127, 128, 129, 256, 300, 384, 385, 1000])
def test_attention_flops_count_every_visible_key(T):
    H, HD = 4, 64
    chunks, _ = _chunk_loop(T)
    keys = readout_tokens = 0
    for s, tc, prev, bank in chunks:
        for j in range(tc):                      # token j of the chunk sees keys 0..j of its own chunk
            keys += j + 1 + (C if prev else 0) + ((SINKS + S) if bank else 0)
        readout_tokens += tc if bank else 0      # M_res exists from the first consolidation on
    assert R.attend_flops(T, H, HD) == 4 * HD * H * keys + 2 * HD * HD * H * readout_tokens


def test_projection_flops_follow_the_layer_shapes():
    cfg = layer_cfg("qwen3_4b")
    D, H, HKV, HD = cfg["dim"], cfg["num_heads"], cfg["num_kv_heads"], cfg["head_dim"]
    # q_proj D -> H*HD, k_proj and v_proj D -> HKV*HD (bolt3.py:33-35), beta_proj D -> HKV (:46),
    # eta_proj D -> H (:49)
    outs = [H * HD, HKV * HD, HKV * HD, HKV, H]
    assert R.proj_in_flops(D, H, HKV, HD) == sum(2 * D * n for n in outs)
    assert R.proj_out_flops(D, H, HD) == 2 * H * HD * D


def test_headline_totals_are_pinned():
    cfg = layer_cfg("qwen3_4b")
    D, H, HKV, HD = cfg["dim"], cfg["num_heads"], cfg["num_kv_heads"], cfg["head_dim"]
    pre = R.prefill_flops(8, 8192, D, H, HKV, HD)           # configs[1]
    assert pre["total"] == sum(v for k, v in pre.items() if k != "total")
    assert pre["total"] == 3_974_321_143_808
    assert pre["consolidate"] == 8 * HKV * 62 * 7 * 2 * C * S * HD
    dec = R.decode_step_bytes(256, D, H, HKV, HD)           # configs[2]
    assert dec == {"state": 485_761_024, "weights": 52_633_600, "total": 538_394_624}
    # the weights: the fused input projection and o_proj in bf16, read once per step
    assert dec["weights"] == 2 * (D * (H * HD + 2 * HKV * HD + HKV + H) + H * HD * D)


def test_decode_state_bytes_cover_the_state_read_per_step():
    # every term of the per-sequence state against the arrays a step reads (include/bolt3.h layouts)
    HKV, HD = 8, 128
    bank = 2 * HKV * S * HD * 2 + HKV * S * (4 + 1)         # ak_rope + av (bf16), mass (fp32) + act (u8)
    m_res = HKV * HD * HD * 4
    sinks = 2 * HKV * SINKS * HD * 2
    window = 2 * HKV * (C + (C + 1) / 2) * HD * 2           # previous chunk + half of the current one
    new = 3 * HKV * HD * 2 + HKV * 4                        # k_raw, k_rope, v of the new token, beta
    per_seq_read = bank + m_res + sinks + window + new
    state = R.decode_step_bytes(1, 2560, 32, HKV, HD, with_weights=False)["state"]
    cons = state - per_seq_read                             # the consolidation, amortised over C steps
    assert 0 < cons < 0.1 * state
