"""Q3_LUT weights (BlockQ3_LUT, codon-infer src/lib.rs:1288-1514): the product's host quantizer
against the oracle's restatement and against a third, scalar float32 restatement in numpy (all
three follow the reference's order of f32 operations), the reference's own round-trip test, the
truncating f32->f16 scale encoding, and the Q3_LUT model layout (Q4_0 attention matrices, Q3_LUT
fc1 / fc2). CPU only."""
import numpy as np
import pytest

LEVELS = [np.float32(v) for v in (0.0955, 0.3030, 0.5496, 0.8849)]  # CENTROIDS_Q3, src/lib.rs:1339


def f32_to_f16_ref(v):
    # f32_to_f16, src/lib.rs:1291-1312.
    bits = int(np.array([v], dtype=np.float32).view(np.uint32)[0])
    sign, exp, frac = (bits >> 31) & 1, (bits >> 23) & 0xFF, bits & 0x7FFFFF
    if exp == 0:
        return sign << 15
    if exp == 0xFF:
        return (sign << 15) | 0x7C00 | min(frac >> 13, 0x3FF)
    e = exp - 127 + 15
    if e >= 31:
        return (sign << 15) | 0x7C00
    if e <= 0:
        return sign << 15
    return (sign << 15) | (e << 10) | (frac >> 13)


def f16_to_f32_ref(h):
    # f16_to_f32, src/lib.rs:1314-1337.
    sign = (h >> 15) << 31
    exp, frac = (h >> 10) & 0x1F, h & 0x3FF
    if exp == 0:
        if frac == 0:
            bits = sign
        else:
            shift = 0
            while (frac & 0x400) == 0:
                frac <<= 1
                shift += 1
            bits = sign | ((127 - 15 + 1 - shift) << 23) | ((frac & 0x3FF) << 13)
    elif exp == 31:
        bits = sign | 0x7F800000 | (frac << 13)
    else:
        bits = sign | ((exp + 127 - 15) << 23) | (frac << 13)
    return np.array([bits], dtype=np.uint32).view(np.float32)[0]


def quantize_block_np(x):
    """BlockQ3_LUT::quantize (src/lib.rs:1355-1458) in scalar numpy float32 arithmetic."""
    f = np.float32
    x = [f(v) for v in x]
    signs, mags, max_abs, sum_sq = 0, [], f(0), f(0)
    for i, v in enumerate(x):
        if v < 0:
            signs |= 1 << i
        a = abs(v)
        mags.append(a)
        if a > max_abs:
            max_abs = a
        sum_sq = f(sum_sq + f(a * a))
    if max_abs < f(1e-8):
        return bytes(14)
    rms = np.sqrt(f(sum_sq / f(32.0)))
    starts = [f(max_abs / LEVELS[3]), max_abs, f(rms * f(2.2)), f(rms * f(1.6))]

    def nearest(m, s):
        bk, md = 0, abs(f(m - f(s * LEVELS[0])))
        for k in range(1, 4):
            dk = abs(f(m - f(s * LEVELS[k])))
            if dk < md:
                bk, md = k, dk
        return bk

    best_err, best_half, best_idx = f(np.finfo(np.float32).max), 0, [0] * 32
    for s0 in starts:
        s = max(s0, f(1e-8))
        for _ in range(4):
            num, den = f(0), f(0)
            idx = [nearest(m, s) for m in mags]
            for m, k in zip(mags, idx):
                num = f(num + f(m * LEVELS[k]))
                den = f(den + f(LEVELS[k] * LEVELS[k]))
            if den > f(1e-8):
                s = f(num / den)
        half = f32_to_f16_ref(s)
        sq = f16_to_f32_ref(half)
        idx = [nearest(m, sq) for m in mags]
        err = f(0)
        for m, k in zip(mags, idx):
            diff = f(m - f(sq * LEVELS[k]))
            err = f(err + f(diff * diff))
        if err < best_err:
            best_err, best_half, best_idx = err, half, idx
    out = bytearray(14)
    out[0:4] = signs.to_bytes(4, "little")
    for b in range(8):
        out[4 + b] = (best_idx[4 * b] | (best_idx[4 * b + 1] << 2) | (best_idx[4 * b + 2] << 4)
                      | (best_idx[4 * b + 3] << 6))
    out[12:14] = best_half.to_bytes(2, "little")
    return bytes(out)


def sample_blocks(rng, nblocks):
    x = (rng.standard_normal((nblocks, 32)) * rng.choice([1e-3, 0.02, 1.0, 50.0], (nblocks, 1))).astype(np.float32)
    x[0] = 0.0                                   # below 1e-8: all-zero block
    x[1] = np.float32(3e-9)                      # still below the threshold
    x[2] = (np.arange(32) / 31.0 * 2 - 1)        # the reference's round-trip block
    x[3, 5] = 1e5                                # scale beyond the half range
    x[4] = np.abs(x[4])                          # no negative signs
    return x


@pytest.mark.parametrize("seed", [0, 1])
def test_q3_quantizer_matches_oracle(esm, orc, seed):
    rng = np.random.default_rng(seed)
    x = sample_blocks(rng, 8192).ravel()
    np.testing.assert_array_equal(esm.quantize_q3(x), orc.quantize_q3(x))


def test_q3_quantizer_matches_scalar_restatement(esm):
    rng = np.random.default_rng(5)
    x = sample_blocks(rng, 48)
    got = esm.quantize_q3(x.ravel()).reshape(-1, 14)
    for b in range(x.shape[0]):
        assert got[b].tobytes() == quantize_block_np(x[b]), f"block {b}"


def test_q3_round_trip_cosine(orc):
    # test_q3_lut_quantization_roundtrip, src/lib.rs:6852-6863.
    src = (np.arange(32) / 31.0 * 2.0 - 1.0).astype(np.float32)
    blocks = orc.quantize_q3(src)
    assert blocks.size == 14
    dst = orc.dequantize_q3(blocks)
    cos = float(np.dot(src, dst) / (np.linalg.norm(src) * np.linalg.norm(dst)))
    assert cos > 0.98


def test_q3_half_encoding_known_answers():
    # The reference truncates the mantissa and has no subnormal halves.
    assert f32_to_f16_ref(np.float32(1.0)) == 0x3C00
    assert f32_to_f16_ref(np.float32(-2.5)) == 0xC100
    assert f32_to_f16_ref(np.float32(65520.0)) == 0x7BFF      # IEEE rounding would give infinity
    assert f32_to_f16_ref(np.float32(1e-5)) == 0x0000         # would be a subnormal half
    assert f32_to_f16_ref(np.float32(1e6)) == 0x7C00
    assert f16_to_f32_ref(0x3C00) == np.float32(1.0)
    assert f16_to_f32_ref(0x0001) == np.float32(2.0 ** -24)   # subnormal halves decode exactly


def test_q3_model_layout_and_dequant(esm, orc):
    # EsmWeights::quantize_q3 (src/lib.rs:609-633): Q4_0 attention matrices, Q3_LUT fc1 / fc2; the
    # oracle's decode of the product's blocks reproduces the reference's LUT values.
    cfg = esm.EsmConfig(64, 256, 1, 4, arch=0)
    t = esm.quantize_tensors(esm.synth_fp32_tensors(cfg, seed=2), esm.DTYPE_Q3_LUT)
    assert t["wq"].size == 64 * 64 // 32 * 20 and t["fc1_w"].size == 256 * 64 // 32 * 14
    vals = orc.dequantize_q3(t["fc1_w"])
    s = vals.reshape(-1, 32)
    assert np.isfinite(vals).all() and (np.abs(s) > 0).any()
