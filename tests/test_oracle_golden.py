"""The oracle pinned against the reference's own golden vectors and tests.

tests/golden/ holds fixtures produced from the reference by make_golden.py:
tests/vectors.json (crates/needle-core/tests/parity_tests.rs) and the numpy
packer tools/export.py:56-84.  Tolerances are the reference tests' own.
"""
import json
import os

import numpy as np
import pytest

import oracle as orc
from conftest import GOLDEN

V = json.load(open(os.path.join(GOLDEN, "tiny_vectors.json")))
TOL = 1e-5  # parity_tests.rs:18


def test_sign_extend_kat():
    # quant.rs:426-431
    assert orc.lib().orc_sign_extend4(0x7) == 7
    assert orc.lib().orc_sign_extend4(0x8) == -8
    assert orc.lib().orc_sign_extend4(0xF) == -1
    assert orc.lib().orc_sign_extend4(0x0) == 0


def test_quantization_vectors():
    # parity_tests.rs:237-263: scales within 1e-6; codes are the reference's
    # w_quantized_int exactly.
    q = V["quantization"]
    w = np.array(q["w"], np.float32)
    data, scales = orc.quantize(w)
    want_s = np.array(q["scales"], np.float32)
    assert scales.shape == want_s.shape
    assert np.max(np.abs(scales - want_s)) < 1e-6
    codes = np.array(q["w_quantized_int"], np.float32)
    lo = ((data & 0x0F).astype(np.int8) << 4) >> 4
    hi = (data.astype(np.int8)) >> 4
    got = np.empty((w.shape[0], w.shape[1]), np.int8)
    got[0::2] = lo.reshape(-1, w.shape[1])
    got[1::2] = hi.reshape(-1, w.shape[1])
    np.testing.assert_array_equal(got.astype(np.float32), codes)


def test_packing_kat_bit_exact():
    kat = json.load(open(os.path.join(GOLDEN, "packing_kat.json")))
    assert len(kat["cases"]) >= 8
    for c in kat["cases"]:
        w = np.frombuffer(bytes.fromhex(c["w_f32_hex"]), np.float32).reshape(c["in_feat"], c["out_feat"])
        data, scales = orc.quantize(w)
        assert data.tobytes().hex() == c["packed_hex"], (c["in_feat"], c["out_feat"])
        assert scales.tobytes().hex() == c["scales_f32_hex"], (c["in_feat"], c["out_feat"])


def test_round_half_away_from_zero():
    # quant.rs:113 uses libm roundf: .5 ties go away from zero.
    w = np.zeros((32, 1), np.float32)
    w[:6, 0] = [7.0, 0.5, 1.5, 2.5, -0.5, -2.5]  # scale = 7/7 = 1 exactly
    data, scales = orc.quantize(w)
    assert scales[0, 0] == 1.0
    deq = orc.dequantize(data, scales, 32, 1)[:6, 0]
    np.testing.assert_array_equal(deq, [7, 1, 2, 3, -1, -3])


def test_roundtrip_identity():
    # quant.rs:434-451
    i, o = np.meshgrid(np.arange(64), np.arange(32), indexing="ij")
    w = ((i + o) % 8).astype(np.float32)
    data, scales = orc.quantize(w)
    out = orc.dequantize(data, scales, 64, 32)
    assert np.max(np.abs(out - w)) < 1e-5


@pytest.mark.parametrize("path", [0, 1])
def test_matvec_matches_dequantize(path):
    # quant.rs:454-489
    w = ((np.arange(64 * 32, dtype=np.float32) - 32.0) * 0.05).reshape(64, 32)
    x = np.sin(np.arange(64, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    data, scales = orc.quantize(w)
    dq = orc.dequantize(data, scales, 64, 32)
    y_ref = x.astype(np.float64) @ dq.astype(np.float64)
    y = orc.matmul(data, scales, 64, 32, x, path)[0]
    assert np.all(np.abs(y - y_ref) < 1e-3 * np.maximum(np.abs(y_ref), 1.0))


@pytest.mark.parametrize("in_feat,out_feat", [(33, 8), (65, 16)])
def test_quant_nonaligned_infeats(in_feat, out_feat):
    # parity_tests.rs:640-676
    w = (np.arange(in_feat * out_feat, dtype=np.float32) * np.float32(0.13) - 4.0).reshape(in_feat, out_feat)
    data, scales = orc.quantize(w)
    assert scales.shape[0] == (in_feat + 31) // 32
    dq = orc.dequantize(data, scales, in_feat, out_feat)
    x = np.sin(np.arange(in_feat, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    y_ref = x.astype(np.float64) @ dq.astype(np.float64)
    for path in (0, 1):
        y = orc.matmul(data, scales, in_feat, out_feat, x, path)[0]
        assert np.all(np.abs(y - y_ref) < 1e-3 * np.maximum(np.abs(y_ref), 1.0))


def test_avx2_and_scalar_paths_agree_closely():
    rng = np.random.default_rng(0)
    w = rng.standard_normal((512, 72)).astype(np.float32)
    x = rng.standard_normal((3, 512)).astype(np.float32)
    data, scales = orc.quantize(w)
    a = orc.matmul(data, scales, 512, 72, x, 0)
    b = orc.matmul(data, scales, 512, 72, x, 1)
    assert np.max(np.abs(a - b)) < 1e-4


def test_quant_matvec_roundtrip():
    # parity_tests.rs:183-196
    w = ((np.arange(16, dtype=np.float32) - 7.5) * np.float32(0.9)).reshape(4, 4)
    data, scales = orc.quantize(w)
    y = orc.matmul(data, scales, 4, 4, np.array([1, 0, 0, 0], np.float32))[0]
    dq = orc.dequantize(data, scales, 4, 4)
    assert np.max(np.abs(y - dq[0])) < TOL


def test_zc_rms_norm_vectors():
    # parity_tests.rs:67-117 and :201-216
    z = V["zc_rms_norm"]
    x = np.array(z["x"], np.float32)
    np.testing.assert_allclose(orc.zc_rms_norm(x, z["scale_zero"]), z["out_zero"], atol=TOL, rtol=0)
    np.testing.assert_allclose(orc.zc_rms_norm(x, z["scale_nonzero"]), z["out_nonzero"], atol=TOL, rtol=0)
    tiny = orc.zc_rms_norm(np.full(4, 1e-4, np.float32), np.zeros(4, np.float32))
    assert tiny[0] < 1.0  # eps inside the sqrt


def test_rope_vectors():
    # parity_tests.rs:120-149 and :218-235
    r = V["rope"]
    hd = r["head_dim"]
    c, s = orc.rope_table(8, hd)
    np.testing.assert_allclose(c[0], r["cos_table_pos0"], atol=TOL, rtol=0)
    np.testing.assert_allclose(s[0], r["sin_table_pos0"], atol=TOL, rtol=0)
    np.testing.assert_allclose(c[1], r["cos_table_pos1"], atol=TOL, rtol=0)
    np.testing.assert_allclose(s[1], r["sin_table_pos1"], atol=TOL, rtol=0)
    q = np.array(r["q_before"], np.float32)
    np.testing.assert_allclose(orc.rope_apply(q, 1, 1, hd, 0), r["q_after_pos0"], atol=TOL, rtol=0)
    got = orc.rope_apply(np.array([1, 2, 3, 4], np.float32), 1, 1, 4, 1)
    c0, s0, c1, s1 = np.cos(1.0), np.sin(1.0), np.cos(0.01), np.sin(0.01)
    want = [1 * c0 - 3 * s0, 2 * c1 - 4 * s1, 3 * c0 + 1 * s0, 4 * c1 + 2 * s1]
    np.testing.assert_allclose(got, want, atol=TOL, rtol=0)


def test_kv_cache_saturates_at_max_len():
    # parity_tests.rs:156-178
    assert orc.lib().orc_kv_cache_push_count(4, 4) == 4
    assert orc.lib().orc_kv_cache_push_count(4, 6) == 4


def test_softmax_guards():
    # ops.rs:5-36: all -inf -> uniform
    np.testing.assert_allclose(orc.softmax([-np.inf] * 4), [0.25] * 4)
    np.testing.assert_allclose(orc.softmax([0.0, 0.0]), [0.5, 0.5])


@pytest.fixture(scope="module")
def tiny():
    return orc.Model(os.path.join(GOLDEN, "tiny_model.safetensors"))


def test_tiny_config(tiny):
    c = V["config"]
    assert tiny.cfg["d_model"] == c["d_model"] and tiny.cfg["vocab_size"] == c["vocab_size"]
    assert tiny.cfg["num_heads"] == c["num_heads"] and tiny.cfg["num_kv_heads"] == c["num_kv_heads"]


def test_full_forward_pred_token_exact(tiny):
    # parity_tests.rs:399-440 (pred_token_q) and :345-397 (pred_token)
    enc, lg = tiny.forward(V["inputs"]["enc_ids"], [V["inputs"]["dec_start_id"]])
    pred = int(np.argmax(lg[0]))
    assert pred == V["forward"]["pred_token_q"]
    assert pred == V["forward"]["pred_token"]


def test_full_forward_logits_quant_close(tiny):
    # parity_tests.rs:442-486 (tol 0.05)
    _, lg = tiny.forward(V["inputs"]["enc_ids"], [V["inputs"]["dec_start_id"]])
    assert np.max(np.abs(lg[0] - np.array(V["forward"]["logits_q"], np.float32))) < 0.05


def test_full_forward_logits_close(tiny):
    # parity_tests.rs:596-637 (INT4 vs f32 python, tol 1.0)
    _, lg = tiny.forward(V["inputs"]["enc_ids"], [V["inputs"]["dec_start_id"]])
    assert np.max(np.abs(lg[0] - np.array(V["forward"]["logits"], np.float32))) < 1.0


def test_encoder_hidden_parity(tiny):
    # parity_tests.rs:488-528 (tol 0.05)
    enc, _ = tiny.forward(V["inputs"]["enc_ids"], [])
    want = np.array(V["forward"]["enc_out_q"], np.float32).reshape(enc.shape)
    assert np.max(np.abs(enc - want)) < 0.05


def test_multi_step_decode_parity(tiny):
    # parity_tests.rs:530-594: exact when margin > 0.05, else in top-5.
    steps = V["multi_step"]["steps"]
    ids, margins = tiny.generate(V["inputs"]["enc_ids"], len(steps), stop_on_eos=False)
    for got, st in zip(ids, steps):
        if st["margin"] > 0.05:
            assert got == st["pred_token"]
        else:
            assert got in st["top5_tokens"]


def test_generate_stops_on_eos(tiny):
    # engine.rs:306-308: EOS (1) ends generation and is not emitted.
    ids, _ = tiny.generate(V["inputs"]["enc_ids"], 8, stop_on_eos=True)
    assert 1 not in ids.tolist()


def test_bad_weights_rejected():
    with pytest.raises(ValueError):
        orc.Model(data=b"\x01\x00")
    with pytest.raises(ValueError):
        orc.Model(data=(100).to_bytes(8, "little") + b"{}")
