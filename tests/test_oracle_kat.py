"""The CPU oracle pinned to every known-answer test the reference holds for
this path (citations are objeta repository paths)."""
import math

import numpy as np
import pytest

from oracle import oracle as O


def test_fp4_nibble_order():
    # crates/objeta-cuda/src/quant.rs:1859-1870
    block = np.zeros(32, np.float32)
    block[0], block[1], block[2] = 0.5, 1.5, 6.0
    d = O.quantize_block(O.FP4_E2M1, block)
    assert d[0] == 127
    assert d[1] == 1 | (3 << 4)


def test_fp4_positive_negative_values():
    # quant.rs:1872-1884
    block = np.zeros(32, np.float32)
    block[0], block[1], block[2], block[3] = 6.0, -6.0, 2.0, -2.0
    d = O.quantize_block(O.FP4_E2M1, block)
    assert d[0] == 127
    assert d[1] == 7 | (15 << 4)
    assert d[2] == 4 | (12 << 4)


def test_fp4_multiple_scale_blocks():
    # quant.rs:1886-1900 (values built with f32 arithmetic as in the test)
    m = np.zeros(128, np.float32)
    for i in range(32):
        m[i] = np.float32(i) / np.float32(32.0) * np.float32(6.0)
    for i in range(32, 64):
        m[i] = np.float32(i - 32) / np.float32(32.0) * np.float32(12.0)
    q = O.quantize_matrix(O.FP4_E2M1, m, 2, 64)
    assert q[0] == 127
    assert q[17] == 128


@pytest.mark.parametrize("fmt", [O.Q4_0, O.IQ3_0, O.FP4_E2M1, O.Q5_0])
def test_rejects_non_multiple_cols(fmt):
    # quant.rs:1664-1670, 1801-1807, 1902-1908
    with pytest.raises(ValueError, match="multiple of block_size"):
        O.quantize_matrix(fmt, np.zeros(4 * 33, np.float32), 4, 33)


def test_fp4_decode_synthetic_fixture():
    # crates/objeta-parser/src/deepseek.rs:1292-1334 (block_size 4)
    out = O.fp4_decode_split(np.array([0x21, 0x43, 0x65, 0x97], np.uint8),
                             np.array([130, 131], np.uint8), 2, 4, 4)
    assert out.tolist() == [4.0, 8.0, 12.0, 16.0, 48.0, 64.0, 96.0, -8.0]


def test_fp4_decode_code8_is_positive_zero():
    # deepseek.rs:789-792: the parser table decodes code 8 to +0.0
    out = O.fp4_decode_split(np.array([0x88], np.uint8), np.array([127], np.uint8), 1, 2, 2)
    assert out[0] == 0.0 and not math.copysign(1.0, float(out[0])) < 0


def test_f8e8m0_to_f32():
    # deepseek.rs:1337-1348
    assert O.f8e8m0_to_f32(127) == 1.0
    assert O.f8e8m0_to_f32(128) == 2.0
    assert O.f8e8m0_to_f32(130) == 8.0
    assert O.f8e8m0_to_f32(126) == 0.5
    assert O.f8e8m0_to_f32(124) == 0.125
    tiny = O.f8e8m0_to_f32(0)
    assert 0.0 < tiny < 1e-38
    assert O.f8e8m0_to_f32(255) == math.inf


def test_e8m0_decoders_agree():
    # quant.rs:886-892 and deepseek.rs:831-850 give the same value for all codes
    for r in range(256):
        a, b = O.decode_f8_e8m0(r), O.f8e8m0_to_f32(r)
        assert a == b, r


def test_f8e4m3_decode():
    # deepseek.rs:1351-1357
    assert abs(O.f8e4m3_to_f32(0x38) - 1.0) < 0.01
    assert O.f8e4m3_to_f32(0x00) == 0.0


def test_cpu_router_top_k_selection():
    # crates/objeta-cuda/src/bin/deepseek_single_layer_moe.rs:3414-3445
    hidden, n, k = 4, 4, 2
    router = np.zeros(n * hidden, np.float32)
    router[1 * hidden:2 * hidden] = 1.0
    router[3 * hidden:4 * hidden] = 2.0
    ids, w = O.router(router, np.full(hidden, 0.5, np.float32), n, hidden, k)
    assert ids.tolist() == [3, 1]
    assert w[0] > w[1]


def test_router_ties_keep_lower_index():
    # stable sort_by (deepseek_single_layer_moe.rs:735): equal probs keep order
    ids, _ = O.router_from_logits(np.array([1.0, 2.0, 2.0, 0.5, 2.0], np.float32), 3)
    assert ids.tolist() == [1, 2, 4]


def test_router_renormalize():
    ids, w = O.router_from_logits(np.array([0.1, 0.9, 0.3, 0.2], np.float32), 2, renormalize=True)
    assert ids.tolist() == [1, 2]
    assert abs(float(w.sum()) - 1.0) < 1e-6


def test_f16_codec_matches_reference_rounding():
    # quant.rs:1046-1079: add one when mantissa bit 12 is set
    assert O.f32_to_f16_bits(1.0) == 0x3C00
    assert O.f32_to_f16_bits(-2.0) == 0xC000
    assert O.f32_to_f16_bits(65504.0) == 0x7BFF
    assert O.f32_to_f16_bits(1e6) == 0x7C00
    assert O.f32_to_f16_bits(float("inf")) == 0x7C00
    assert O.f32_to_f16_bits(float("nan")) == 0x7E00
    # 1 + 2^-11 (bit 12 set exactly): reference rounds up, RNE would not
    v = np.float32(1.0) + np.float32(2.0 ** -11)
    assert O.f32_to_f16_bits(float(v)) == 0x3C01
    # subnormal half and underflow
    assert O.f32_to_f16_bits(2.0 ** -24) == 0x0001
    assert O.f32_to_f16_bits(2.0 ** -40) == 0x0000
    for bits in (0x0001, 0x03FF, 0x0400, 0x3C00, 0x7BFF, 0x8001, 0xFBFF):
        f = O.f16_to_f32_bits(bits)
        assert f == float(np.array([bits], np.uint16).view(np.float16)[0])


def test_f16_decode_exhaustive_vs_numpy():
    codes = np.arange(65536, dtype=np.uint16)
    ref = codes.view(np.float16).astype(np.float32)
    got = np.array([O.f16_to_f32_bits(int(c)) for c in codes[::7]], np.float32)
    r = ref[::7]
    fin = np.isfinite(r)
    assert np.array_equal(got[fin], r[fin])
    assert np.all(np.isnan(got[np.isnan(r)]))


def test_seeded_f32s_lcg():
    # quant.rs:1610-1620: first value from seed 0: state = 1 -> bits = 1
    v = O.seeded_f32s(3, 0)
    assert v[0] == np.float32(np.float32(1.0) / np.float32(4294967295.0) * np.float32(2.0) - np.float32(1.0))
    assert np.all(np.abs(O.seeded_f32s(1000, 123)) <= 1.0)


def test_q4_roundtrip_small_cosine():
    # quant.rs:1672-1692 (q4_cpu_reference_roundtrip_small)
    m = O.seeded_f32s(16 * 32, 42)
    x = O.seeded_f32s(32, 7)
    q = O.quantize_matrix(O.Q4_0, m, 16, 32)
    r = O.gemv(O.Q4_0, q, x, 16, 32)
    d = O.dense_gemv(m, x, 16, 32)
    assert O.compare_outputs(d, r)["cosine_similarity"] > 0.995


def test_q5_no_worse_than_q4():
    # quant.rs:1767-1799
    rows, cols, seed = 128, 256, 77
    m = O.seeded_f32s(rows * cols, seed ^ 0x1234_5678_9ABC_DEF0)
    x = O.seeded_f32s(cols, seed ^ 0x0BAD_F00D_1234_5678)
    d = O.dense_gemv(m, x, rows, cols)
    q4 = O.compare_outputs(d, O.gemv(O.Q4_0, O.quantize_matrix(O.Q4_0, m, rows, cols), x, rows, cols))
    q5 = O.compare_outputs(d, O.gemv(O.Q5_0, O.quantize_matrix(O.Q5_0, m, rows, cols), x, rows, cols))
    assert q5["cosine_similarity"] >= q4["cosine_similarity"] - 1e-6
    assert q5["relative_l2_error"] <= q4["relative_l2_error"] + 1e-6


def test_iq3_roundtrip_small_cosine():
    # quant.rs:1809-1828
    m = O.seeded_f32s(16 * 32, 44)
    x = O.seeded_f32s(32, 9)
    q = O.quantize_matrix(O.IQ3_0, m, 16, 32)
    assert O.compare_outputs(O.dense_gemv(m, x, 16, 32), O.gemv(O.IQ3_0, q, x, 16, 32))[
        "cosine_similarity"] > 0.970


def test_native_fp4_expert_bytes():
    # moe.rs:2474-2478: 6 tensors of a 256/512/256 expert = 208896 bytes
    h, i, o = 256, 512, 256
    assert (i * h // 2) * 2 + (i * h // 32) * 2 + (o * i // 2) + (o * i // 32) == 208896


# ---------------------------------------------- official DeepSeek path (deepseek.rs)
def test_act_quant_fixture():
    """deepseek.rs:1382-1394 (test_act_quant_fixture): block 8, scales 127 and 120."""
    x = np.array([1.0, 448.0, -448.0, 0.0, 100.0, 200.0, -100.0, -200.0,
                  1.0, 2.0, 0.5, -0.5, 0.0, 0.0, 0.0, 0.0], np.float32)
    y, s = O.act_quant(x, 8)
    assert y.size == 16 and s.size == 2
    assert s.tolist() == [127, 120]


def test_f32_to_f8e4m3_exact_codes():
    """deepseek.rs:1444-1481: the encoder's branches, and decode(encode(v)) == v
    for every normal E4M3 value (exponent fields 1..14)."""
    enc = O.f32_to_f8e4m3_exact
    assert enc(1.0) == 0x38 and enc(2.0) == 0x40 and enc(3.0) == 0x44 and enc(4.0) == 0x48
    assert enc(448.0) == 0x7E and enc(-1000.0) == 0xFE
    assert enc(0.001) == 0 and enc(-0.001) == 0x80         # below 2^-7: flushed (signed)
    assert enc(1.5 / 128) == 0x04                           # [2^-7, 2^-6): exponent field 0
    for c in range(256):
        e = (c >> 3) & 15
        if 1 <= e <= 14:
            v = O.f8e4m3_to_f32(c)
            assert enc(v) == c, hex(c)


def test_fp8_fp4_gemv_oracle_small_case():
    """Hand-checked: act = [1, 2] * 2^0 (codes 0x38, 0x40), weights +1 / -0.5."""
    act = np.zeros(128, np.uint8)
    act[0], act[1] = 0x38, 0x40
    act_s = np.array([127], np.uint8)
    w = np.zeros(64, np.uint8)
    w[0] = 0x2 | (0x9 << 4)               # codes 2 (+1.0) and 9 (-0.5)
    ws = np.full(4, 127, np.uint8)
    y = O.fp8_act_fp4_weight_gemv_f32(act, act_s, w, ws, 1, 128)
    assert y[0] == np.float32(1.0 * 1.0 + 2.0 * -0.5)


# ------------------------------------------------------ DeepSeek gate (dsl_moe.rs:883-1000)
def test_gate_sqrtsoftplus_scores():
    ids, w = O.deepseek_gate(np.zeros(256 * 4096), np.full(4096, 0.1), 256, 4096, 6, O.SQRT_SOFTPLUS, 1.5)
    assert ids.size == 6 and abs(float(w.sum()) - 1.5) < 1e-4
    assert ids.tolist() == [0, 1, 2, 3, 4, 5]            # equal scores: the stable sort keeps index order


def test_gate_bias_affects_selection_not_weights():
    gate = np.zeros(256 * 4096, np.float32)
    gate[0] = 1.0
    ids, _ = O.deepseek_gate(gate, np.ones(4096), 256, 4096, 6, O.SQRT_SOFTPLUS, 1.5, gate_bias=np.zeros(256))
    assert 0 in ids.tolist()
    bias = np.zeros(256, np.float32)
    bias[7] = 100.0
    ids2, w2 = O.deepseek_gate(gate, np.ones(4096), 256, 4096, 6, O.SQRT_SOFTPLUS, 1.5, gate_bias=bias)
    assert ids2[0] == 7 and abs(float(w2.sum()) - 1.5) < 1e-4


def test_gate_hash_layer_tid2eid():
    tid2eid = np.arange(129280 * 6) % 256
    ids, w = O.deepseek_gate(np.zeros(256 * 4096), np.full(4096, 0.1), 256, 4096, 6, O.SQRT_SOFTPLUS, 1.5,
                             tid2eid=tid2eid, input_id=42)
    assert ids.tolist() == tid2eid[42 * 6:43 * 6].tolist() and abs(float(w.sum()) - 1.5) < 1e-4
    import pytest
    with pytest.raises(ValueError):
        O.deepseek_gate(np.zeros(256 * 4096), np.full(4096, 0.1), 256, 4096, 6, O.SQRT_SOFTPLUS, 1.5,
                        tid2eid=tid2eid, input_id=129280)


def test_gate_hash_layer_weights_from_hidden():
    gate = np.zeros((256, 4096), np.float32)
    gate[0] = 0.5
    gate[100] = 2.0
    tid2eid = np.arange(129280 * 6) % 256
    ia, wa = O.deepseek_gate(gate, np.ones(4096), 256, 4096, 6, O.SQRT_SOFTPLUS, 1.5, tid2eid=tid2eid, input_id=0)
    ib, wb = O.deepseek_gate(gate, -np.ones(4096), 256, 4096, 6, O.SQRT_SOFTPLUS, 1.5, tid2eid=tid2eid, input_id=0)
    assert ia.tolist() == [0, 1, 2, 3, 4, 5] and ib.tolist() == ia.tolist()
    assert not np.array_equal(wa, wb)


def test_gate_route_scale_and_top_k():
    _, w = O.deepseek_gate(np.zeros(256 * 4096), np.full(4096, 0.42), 256, 4096, 6, O.SQRT_SOFTPLUS, 1.5)
    assert abs(float(w.sum()) - 1.5) < 1e-4
    gate = np.zeros((256, 4096), np.float32)
    gate[10], gate[20], gate[30] = 3.0, 2.0, 1.0
    ids, _ = O.deepseek_gate(gate, np.ones(4096), 256, 4096, 6, O.SQRT_SOFTPLUS, 1.5)
    assert ids[:3].tolist() == [10, 20, 30]
