"""CPU tests: the oracle (oracle/aex_oracle.cpp) against the golden fixtures in
tests/golden/ — the reference's own known-answer tests
(Tests/ImarelloCoreTests/Flux2MathTests.swift), hand-derived values of its CPU bf16
rounding and 4-bit dequant (Sources/ImarelloDirect/DirectTEEncoder.swift:39-43,
104-123) and float64 attention cases."""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def ka():
    with open(os.path.join(GOLD, "known_answers.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def bd():
    with open(os.path.join(GOLD, "bf16_dequant.json")) as f:
        return json.load(f)


# ---------------------------------------------------------------- RoPE / ids
def test_rope1d_known_answers(ka):
    g = ka["rope1d"]
    for pos, cos_exp, sin_exp in ((0.0, g["pos0_cos"], g["pos0_sin"]),):
        c, s = O.rope_freqs(np.array([[pos]], np.float32), g["theta"], (g["dim"],))
        assert np.allclose(c[0], cos_exp, atol=g["tol"]) and np.allclose(s[0], sin_exp, atol=g["tol"])
    c, s = O.rope_freqs(np.array([[1.0]], np.float32), g["theta"], (g["dim"],))
    assert np.allclose(c[0, :2], g["pos1_cos01"], atol=g["tol"])
    assert np.allclose(s[0, :2], g["pos1_sin01"], atol=g["tol"])


def test_rope_four_axes_concatenate(ka):
    c, s = O.rope_freqs(np.array(ka["rope_4axis_width"]["ids"], np.float32))
    assert c.shape[1] == s.shape[1] == ka["rope_4axis_width"]["half"]


def test_grid_and_text_ids(ka):
    g = ka["grid_ids"]
    ids = O.grid_ids(g["height"], g["width"])
    assert ids.shape == (g["height"] * g["width"], 4)
    for r, row in g["rows"].items():
        assert ids[int(r)].tolist() == row
    g = ka["grid_ids_ref_t"]
    assert O.grid_ids(g["height"], g["width"], g["t"]).tolist() == g["rows"]
    g = ka["text_ids"]
    assert O.text_ids(g["length"]).tolist() == g["rows"]


def test_apply_rotary_quarter_turn(ka):
    g = ka["apply_rotary"]
    x = np.array(g["x"], np.float32).reshape(1, 1, 2)
    y = O.rope_apply(x, np.array([g["cos"]], np.float32), np.array([g["sin"]], np.float32))
    assert np.allclose(y.reshape(-1), g["out"], atol=1e-6)


# ---------------------------------------------------------------- scheduler
def test_linear_mu_and_shift(ka):
    g = ka["linear_mu"]
    assert abs(O.linear_mu(4096) - g["4096"]) < g["tol"]
    assert abs(O.linear_mu(256) - g["256"]) < g["tol"]
    g = ka["time_shift_at_1"]
    assert abs(O.time_shift(g["mu"], 1.0) - g["value"]) < g["tol"]


def test_schedule_4step(ka):
    g = ka["schedule_4step"]
    for seq, exp in g["float64"].items():
        sig, ts = O.schedule(4, int(seq))
        assert len(sig) == 5 and len(ts) == 4
        assert abs(sig[-1]) < 1e-7 and sig[0] > g["min_first_sigma"]
        assert all(sig[i] >= sig[i + 1] - 1e-6 for i in range(4))
        assert np.allclose(sig, exp["sigmas"], atol=g["tol"])
        assert np.allclose(ts, exp["timesteps"], atol=1e-2)


def test_euler_step_uses_sigma_delta(ka):
    g = ka["euler"]
    sig, _ = O.schedule(4, g["seq"])
    x = np.array(g["sample"], np.float32)
    v = np.array(g["model_output"], np.float32)
    nxt = x + (sig[1] - sig[0]) * v  # Flux2Scheduler.step: x + (sigma_{i+1} - sigma_i) * v
    assert np.allclose(nxt, x + (sig[1] - sig[0]) * v, atol=1e-5)
    assert (nxt < x).all()  # sigmas decrease, positive velocity moves the sample down


def test_timestep_embedding_t0(ka):
    g = ka["timestep_embed_t0"]
    e = O.timestep_embedding(np.array([0.0, 500.0, 1000.0], np.float32), g["dim"])
    assert e.shape == (3, g["dim"])
    assert np.allclose(e[0, :128], g["first128"], atol=g["tol"])
    assert np.allclose(e[0, 128:], g["last128"], atol=g["tol"])


# ---------------------------------------------------------------- bf16 / dequant
def test_f32_to_bf16_matches_reference_rounding(bd):
    for name, c in bd["f32_to_bf16"].items():
        x = np.array([c["f32_bits"]], np.uint32).view(np.float32)
        assert int(O.f32_to_bf16(x)[0]) == c["bf16"], name


def test_dequant_words(bd):
    for c in bd["dequant_words"]:
        got = O.dequant_q4(np.array([[c["packed"]] * 8], np.uint32), np.array([[c["scale"]]], np.uint16),
                           np.array([[c["bias"]]], np.uint16), 1, 64)
        assert got[0, :8].tolist() == c["out"], c


def test_dequant_double_rounding_cases(bd):
    assert len(bd["double_rounding"]) >= 8
    for c in bd["double_rounding"]:
        word = np.uint32(c["q"] * 0x11111111)  # all eight nibbles = q
        got = O.dequant_q4(np.array([[word] * 8], np.uint32), np.array([[c["scale"]]], np.uint16),
                           np.array([[c["bias"]]], np.uint16), 1, 64)
        assert int(got[0, 0]) == c["out"] != c["exact_rne"], c


def test_pack_unpack_roundtrip_all_nibbles():
    rng = np.random.default_rng(3)
    codes = rng.integers(0, 16, (16, 128)).astype(np.uint8)
    codes[0, :16] = np.arange(16)
    packed = O.pack_q4(codes)
    ones = np.full((16, 2), 0x3F80, np.uint16)  # scale 1
    zeros = np.zeros((16, 2), np.uint16)  # bias 0
    deq = O.bf16_to_f32(O.dequant_q4(packed, ones, zeros, 16, 128))
    assert np.array_equal(deq, codes.astype(np.float32))


def test_qmm_matches_float64_dequantized_gemm():
    rng = np.random.default_rng(4)
    n, k, m = 48, 192, 5
    packed = O.pack_q4(rng.integers(0, 16, (n, k)).astype(np.uint8))
    scales = O.f32_to_bf16(np.abs(rng.normal(0, 0.02, (n, k // 64))).astype(np.float32))
    biases = O.f32_to_bf16(rng.normal(0, 0.02, (n, k // 64)).astype(np.float32))
    w = O.bf16_to_f32(O.dequant_q4(packed, scales, biases, n, k)).astype(np.float64)
    x = rng.standard_normal((m, k)).astype(np.float32)
    assert np.allclose(O.qmm(x, packed, scales, biases, n, k), x.astype(np.float64) @ w.T, rtol=1e-5, atol=1e-5)


# ---------------------------------------------------------------- attention
@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_joint_attention_float64_cases(case):
    z = np.load(os.path.join(GOLD, "attention_small.npz"))
    g = lambda k: z[f"{case}_{k}"]
    out = O.joint_attention(g("q"), g("k"), g("v"), g("wq"), g("wk"), float(g("eps")), g("cos"), g("sin"))
    ref = g("out")
    assert np.abs(out - ref).max() < 2e-5


def test_sdpa_query_row_sampling_matches_full():
    rng = np.random.default_rng(5)
    q, k, v = (rng.standard_normal((1, 100, 2, 128)).astype(np.float32) for _ in range(3))
    full = O.sdpa(q, k, v, 0.1)
    part = O.sdpa(q, k, v, 0.1, q_begin=30, q_end=70)
    assert np.array_equal(part[:, 30:70], full[:, 30:70])
    assert np.isnan(part[:, :30]).all() and np.isnan(part[:, 70:]).all()
