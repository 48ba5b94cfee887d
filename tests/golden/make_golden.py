"""Generate the golden fixtures that pin the CPU oracle (oracle/aex_oracle.cpp).

Run from the repository root:  python tests/golden/make_golden.py

Every expected value here is computed independently of the oracle:

* known_answers.json — the reference's own known-answer tests, restated from
  Tests/ImarelloCoreTests/Flux2MathTests.swift (line numbers in each entry), with
  the expected numbers evaluated in float64 from the formulas those tests state.
* bf16_dequant.json — hand-derivable values of the reference's CPU bf16 rounding
  (DirectTEEncoder.f32ToBF16, Sources/ImarelloDirect/DirectTEEncoder.swift:39-43)
  and 4-bit dequant (DirectTEEncoder.embedRow, :104-123), computed with Python
  integers and numpy float32 scalar arithmetic (product rounded, then sum
  rounded, no fused multiply-add), including cases where rounding the exact
  value straight to bf16 would give a different answer (double-rounding cases).
* attention_small.npz — small joint-attention cases (RMSNorm -> interleaved RoPE
  -> softmax(scale QK^T) V, MetalFlashAttentionTests.swift:10-17) evaluated in
  float64 numpy.
"""
import json
import os
import struct
from fractions import Fraction

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def f32_bits(x):
    return struct.unpack("<I", struct.pack("<f", np.float32(x)))[0]


def bits_f32(u):
    return float(struct.unpack("<f", struct.pack("<I", u & 0xFFFFFFFF))[0])


def ref_f32_to_bf16(bits):
    """DirectTEEncoder.f32ToBF16: (bits &+ 0x7FFF &+ ((bits >> 16) & 1)) >> 16, 32-bit wrapping."""
    return (((bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFFFFFF) >> 16) & 0xFFFF


def bf16_f32(u):
    return bits_f32(u << 16)


def dequant_ref(packed_word, scale_bf16, bias_bf16):
    s, b = np.float32(bf16_f32(scale_bf16)), np.float32(bf16_f32(bias_bf16))
    out = []
    for n in range(8):
        q = np.float32((packed_word >> (4 * n)) & 0xF)
        prod = np.float32(s * q)        # rounded to f32
        val = np.float32(prod + b)      # rounded to f32
        out.append(ref_f32_to_bf16(f32_bits(val)))
    return out


def rne_bf16_exact(fr):
    """Round an exact rational straight to bf16 (round-to-nearest-even), for finding double-rounding cases."""
    if fr == 0:
        return 0
    sign = 0x8000 if fr < 0 else 0
    a = abs(fr)
    e = 0
    while a >= 2:
        a /= 2
        e += 1
    while a < 1:
        a *= 2
        e -= 1
    m = a * 128  # 7 fraction bits
    lo = int(m)
    rem = m - lo
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and lo % 2 == 1):
        lo += 1
    if lo == 256:
        lo = 128
        e += 1
    return sign | ((e + 127) << 7) | (lo - 128)


def known_answers():
    theta = 2000.0
    omega1 = 1.0 / theta ** (2.0 / 32.0)
    # Flux2Scheduler formulas (Flux2Scheduler.swift:56-109) in float64
    def mu(seq):
        m = (1.15 - 0.5) / (4096 - 256)
        return m * seq + (0.5 - m * 256)

    def shift(m, t):
        return np.exp(m) / (np.exp(m) + (1.0 / t - 1.0))

    sched = {}
    for seq in (4096, 1024):
        m = mu(seq)
        base = [1.0 + (1.0 / 4 - 1.0) * i / 3 for i in range(4)]
        sig = [shift(m, t) for t in base] + [0.0]
        sched[str(seq)] = {"sigmas": sig, "timesteps": [s * 1000 for s in sig[:4]]}
    return {
        "source": "Tests/ImarelloCoreTests/Flux2MathTests.swift",
        "rope1d": {"lines": "10-29", "dim": 32, "theta": theta,
                   "pos0_cos": [1.0] * 16, "pos0_sin": [0.0] * 16,
                   "pos1_cos01": [float(np.cos(1.0)), float(np.cos(omega1))],
                   "pos1_sin01": [float(np.sin(1.0)), float(np.sin(omega1))], "tol": 1e-5},
        "rope_4axis_width": {"lines": "31-39", "ids": [[0, 1, 2, 3]], "half": 64},
        "grid_ids": {"lines": "41-49", "height": 2, "width": 3,
                     "rows": {"0": [0, 0, 0, 0], "1": [0, 0, 1, 0], "3": [0, 1, 0, 0], "5": [0, 1, 2, 0]}},
        "grid_ids_ref_t": {"lines": "222-228", "height": 1, "width": 2, "t": 10,
                           "rows": [[10, 0, 0, 0], [10, 0, 1, 0]]},
        "apply_rotary": {"lines": "51-56", "x": [1.0, 0.0], "cos": [0.0], "sin": [1.0], "out": [0.0, 1.0]},
        "text_ids": {"lines": "245-251", "length": 3, "rows": [[0, 0, 0, 0], [0, 0, 0, 1], [0, 0, 0, 2]]},
        "timestep_embed_t0": {"lines": "60-72", "dim": 256, "first128": 1.0, "last128": 0.0, "tol": 1e-5},
        "linear_mu": {"lines": "121-127", "4096": 1.15, "256": 0.5, "tol": 1e-5},
        "time_shift_at_1": {"lines": "159-163", "mu": 1.15, "value": 1.0, "tol": 1e-5},
        "schedule_4step": {"lines": "129-142", "min_first_sigma": 0.9, "float64": sched, "tol": 1e-5},
        "euler": {"lines": "144-156", "sample": [1, 2, 3], "model_output": [0.1, 0.1, 0.1], "seq": 1024},
        "image_seq_len": {"lines": "115-119", "cases": [[1024, 1024, 4096], [512, 512, 1024], [768, 512, 1536]]},
    }


def bf16_dequant():
    cases_bits = {
        "one": 0x3F800000, "tie_down_even": 0x3F808000, "tie_up_odd": 0x3F818000, "above_tie": 0x3F808001,
        "below_tie": 0x3F807FFF, "neg": 0xC0200000, "max_finite_rounds_to_inf": 0x7F7FFFFF,
        "smallest_normal": 0x00800000, "denormal": 0x00000001, "neg_zero": 0x80000000,
        "quiet_nan": 0x7FC00001, "all_ones_wraps_to_zero": 0xFFFFFFFF,
    }
    f2b = {k: {"f32_bits": v, "bf16": ref_f32_to_bf16(v)} for k, v in cases_bits.items()}
    rng = np.random.default_rng(1234)
    words = [0x76543210, 0xFEDCBA98, 0x00000000, 0xFFFFFFFF, 0x0F0F0F0F] + [int(w) for w in rng.integers(0, 2**32, 12)]
    scales = [0x3F00, 0x3C23, 0x3A83, 0x3DCC, 0x3B80, 0x0001]  # 0.5, ~0.00995, ~0.001, ~0.0996, ~0.0039, subnormal
    biases = [0xBF80, 0xBC23, 0x3A83, 0x0000, 0x8000, 0xBDCC]
    deq = []
    for w in words:
        for s in scales[:3]:
            for b in biases[:3]:
                deq.append({"packed": w, "scale": s, "bias": b, "out": dequant_ref(w, s, b)})
    # Double-rounding cases: f32(s*q + b) then bf16 differs from bf16 of the exact s*q + b.
    found = []
    for s_bits in range(0x3C00, 0x4100, 7):
        s = bf16_f32(s_bits)
        for q in range(1, 16):
            a = Fraction(s) * q
            for b_bits in (0x8001, 0x8002, 0x0001, 0x0002, 0x3000, 0xB000, 0x2F80, 0xAF80, 0x3380, 0xB380):
                bb = Fraction(bf16_f32(b_bits))
                exact = a + bb
                two_step = ref_f32_to_bf16(f32_bits(np.float32(np.float32(s * q) + np.float32(bf16_f32(b_bits)))))
                if two_step != rne_bf16_exact(exact):
                    found.append({"scale": s_bits, "q": q, "bias": b_bits, "out": two_step,
                                  "exact_rne": rne_bf16_exact(exact)})
            if len(found) >= 24:
                break
        if len(found) >= 24:
            break
    return {"source": "Sources/ImarelloDirect/DirectTEEncoder.swift:39-43,104-123", "f32_to_bf16": f2b,
            "dequant_words": deq, "double_rounding": found}


def attention_cases():
    rng = np.random.default_rng(99)
    out = {}
    for name, (b, s, h, eps) in {"a": (1, 48, 2, 1e-6), "b": (2, 130, 1, 1e-5), "c": (1, 257, 1, 1e-6)}.items():
        q, k, v = (rng.standard_normal((b, s, h, 128)) for _ in range(3))
        wq, wk = (1 + 0.1 * rng.standard_normal(128) for _ in range(2))
        ang = rng.uniform(0, 2 * np.pi, (s, 64))
        cos, sin = np.cos(ang), np.sin(ang)

        def norm(x, w):
            return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * w

        def rope(x):
            re, im = x[..., 0::2], x[..., 1::2]
            c, sn = cos[None, :, None, :], sin[None, :, None, :]
            y = np.empty_like(x)
            y[..., 0::2] = re * c - im * sn
            y[..., 1::2] = im * c + re * sn
            return y

        qn, kn = rope(norm(q, wq)), rope(norm(k, wk))
        sc = np.einsum("bqhd,bkhd->bhqk", qn, kn) / np.sqrt(128)
        sc -= sc.max(-1, keepdims=True)
        p = np.exp(sc)
        p /= p.sum(-1, keepdims=True)
        o = np.einsum("bhqk,bkhd->bqhd", p, v)
        f = lambda a: a.astype(np.float32)
        out.update({f"{name}_q": f(q), f"{name}_k": f(k), f"{name}_v": f(v), f"{name}_wq": f(wq), f"{name}_wk": f(wk),
                    f"{name}_cos": f(cos), f"{name}_sin": f(sin), f"{name}_eps": np.float32(eps), f"{name}_out": f(o)})
    return out


if __name__ == "__main__":
    with open(os.path.join(HERE, "known_answers.json"), "w") as fh:
        json.dump(known_answers(), fh, indent=1)
    with open(os.path.join(HERE, "bf16_dequant.json"), "w") as fh:
        json.dump(bf16_dequant(), fh, indent=1)
    np.savez_compressed(os.path.join(HERE, "attention_small.npz"), **attention_cases())
    print("wrote known_answers.json, bf16_dequant.json, attention_small.npz")
