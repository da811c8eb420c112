"""CPU checks of the oracle's k-quant formats and integer dot (no GPU)."""
import numpy as np
import pytest

from conftest import O, gaussian_qweight


def test_f16_conversions_match_numpy():
    bits = np.arange(0, 65536, 3, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([O.f16_to_f32(int(b)) for b in bits], dtype=np.float32)
    same = (got == ref) | (np.isnan(got) & np.isnan(ref))
    assert same.all()
    rng = np.random.default_rng(3)
    xs = np.concatenate([rng.normal(0, 1, 3000), rng.normal(0, 1e-5, 3000), rng.normal(0, 3e4, 500),
                         [65519.0, 65520.0, 5.96e-8, 2.98e-8, 0.0, -0.0]]).astype(np.float32)
    with np.errstate(over="ignore"):
        want = xs.astype(np.float16).view(np.uint16)
    got = np.array([O.f32_to_f16(float(v)) for v in xs], dtype=np.uint16)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("dtype,bound", [(O.Q4_K, 0.09), (O.Q6_K, 0.025)])
def test_quantize_roundtrip_error(dtype, bound):
    w = np.random.default_rng(0).normal(0, 0.02, (32, 1024)).astype(np.float32)
    q = O.quantize(dtype, w)
    assert q.shape == (32, 1024 // 256 * O.BLOCK_BYTES[dtype])
    dq = O.dequantize(dtype, q, w.size).reshape(w.shape)
    rel = np.linalg.norm(dq - w) / np.linalg.norm(w)
    assert rel < bound


def test_q4k_block_layout_roundtrip():
    """Dequantize follows the GGUF Q4_K layout: d*sc*q - dmin*m with 6-bit
    scales/mins packed as in get_scale_min_k4 (quantized.cu:925-933)."""
    rng = np.random.default_rng(1)
    blk = np.zeros(144, dtype=np.uint8)
    d, dmin = np.float16(0.01), np.float16(0.004)
    blk[0:2] = np.frombuffer(d.tobytes(), np.uint8)
    blk[2:4] = np.frombuffer(dmin.tobytes(), np.uint8)
    sc = rng.integers(0, 64, 8)
    mn = rng.integers(0, 64, 8)
    s = np.zeros(12, dtype=np.int64)
    for j in range(8):
        if j < 4:
            s[j] |= sc[j]
            s[j + 4] |= mn[j]
        else:
            s[j + 4] |= (sc[j] & 0xF) | ((mn[j] & 0xF) << 4)
            s[j - 4] |= (sc[j] >> 4) << 6
            s[j] |= (mn[j] >> 4) << 6
    blk[4:16] = s.astype(np.uint8)
    qv = rng.integers(0, 16, 256)
    for g in range(4):
        for l in range(32):
            blk[16 + 32 * g + l] = qv[64 * g + l] | (qv[64 * g + 32 + l] << 4)
    y = O.dequantize(O.Q4_K, blk, 256)
    want = np.array([np.float32(np.float32(d) * np.float32(sc[i // 32])) * np.float32(qv[i])
                     - np.float32(np.float32(dmin) * np.float32(mn[i // 32])) for i in range(256)], dtype=np.float32)
    assert np.array_equal(y, want)


def test_q8k_quantizer_properties():
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, 2048).astype(np.float32)
    x[300] = -7.0   # negative pivot
    x[1000] = 5.0
    x[1001] = -5.0  # tie in magnitude: the first one is the pivot
    b = O.quantize_q8k(x).reshape(-1, 292)
    for i in range(b.shape[0]):
        d = b[i, :4].view(np.float32)[0]
        qs = b[i, 4:260].view(np.int8).astype(np.int32)
        bs = b[i, 260:292].view(np.int16).astype(np.int32)
        assert np.array_equal(bs, qs.reshape(16, 16).sum(1))
        xb = x[256 * i:256 * (i + 1)]
        piv = xb[np.argmax(np.abs(xb))]
        iscale = np.float32(-128.0) / np.float32(piv)
        assert d == np.float32(1.0) / iscale
        ref = np.minimum(127, np.sign(iscale * xb) * np.floor(np.abs(iscale * xb) + 0.5)).astype(np.int32)
        assert np.array_equal(qs, ref)
    # block 3 holds x[768:1024]... the tie block is block 3 (1000, 1001)
    blk = b[3]
    qs = blk[4:260].view(np.int8)
    assert qs[1000 - 768] == -128 or qs[1000 - 768] == 127  # pivot maps to +-128 (clamped at 127)
    assert qs[1001 - 768] == 127
    zero = O.quantize_q8k(np.zeros(256, np.float32))
    assert not zero.any()


@pytest.mark.parametrize("dtype", [O.Q4_K, O.Q6_K])
def test_integer_dot_equals_dequantized_dot(dtype):
    """sum_j sc_j (q_w . q_x)_j combined with the scales equals the float dot
    of the dequantized operands (the identity the GPU kernel relies on)."""
    k = 2048
    w = gaussian_qweight(dtype, 8, k, seed=11)
    x = np.random.default_rng(12).normal(0, 1, (2, k)).astype(np.float32)
    y = O.qmatmul(dtype, w, 8, k, x)
    wd = O.dequantize(dtype, w, 8 * k).reshape(8, k).astype(np.float64)
    for r in range(2):
        xq = O.quantize_q8k(x[r])
        xd = O.dequantize(O.Q8_K, xq, k).astype(np.float64)
        ref = wd @ xd
        np.testing.assert_allclose(y[r], ref, rtol=1e-5, atol=1e-5)
        for c in range(8):
            assert y[r, c] == O.vec_dot(dtype, k, w[c], xq)


@pytest.mark.parametrize("dtype", [O.Q4_K, O.Q6_K])
def test_block_dots_reconstruct_vec_dot(dtype):
    k = 1024
    w = gaussian_qweight(dtype, 4, k, seed=21)
    x = np.random.default_rng(22).normal(0, 1, k).astype(np.float32)
    xq = O.quantize_q8k(x)
    sc, mn = O.block_dots(dtype, w, 4, k, xq)
    dy = xq.reshape(-1, 292)[:, :4].copy().view(np.float32)[:, 0].astype(np.float64)
    bb = O.BLOCK_BYTES[dtype]
    for r in range(4):
        blocks = w[r].reshape(-1, bb)
        if dtype == O.Q4_K:
            d = blocks[:, 0:2].copy().view(np.float16)[:, 0].astype(np.float64)
            dm = blocks[:, 2:4].copy().view(np.float16)[:, 0].astype(np.float64)
            ref = np.sum(d * dy * sc[r] - dm * dy * mn[r])
        else:
            d = blocks[:, 208:210].copy().view(np.float16)[:, 0].astype(np.float64)
            assert not mn.any()
            ref = np.sum(d * dy * sc[r])
        assert abs(ref - O.vec_dot(dtype, k, w[r], xq)) < 1e-4 * max(1.0, abs(ref))


def test_synth_generators_structure():
    q = O.synth_q4k(5, 64, 0.02).reshape(64, 144)
    dq = O.dequantize(O.Q4_K, q, 64 * 256)
    assert abs(dq.mean()) < 2e-3 and 0.012 < dq.std() < 0.03
    q6 = O.synth_q6k(5, 64, 0.02).reshape(64, 210)
    dq6 = O.dequantize(O.Q6_K, q6, 64 * 256)
    assert 0.01 < dq6.std() < 0.03
    f = O.synth_f32(9, 10000, 1.0, 0.02)
    assert abs(f.mean() - 1.0) < 1e-3 and abs(f.std() - 0.02) < 2e-3
    t = O.synth_tokens(2, 1000, 151936)
    assert t.min() >= 0 and t.max() < 151936
    assert np.array_equal(O.synth_q4k(5, 64, 0.02), O.synth_q4k(5, 64, 0.02))


def test_qmatmul_f32_matches_dequantized_matmul():
    w = gaussian_qweight(O.Q6_K, 16, 512, seed=3)
    x = np.random.default_rng(4).normal(0, 1, (5, 512)).astype(np.float32)
    y = O.qmatmul_f32(O.Q6_K, w, 16, 512, x)
    wd = O.dequantize(O.Q6_K, w, 16 * 512).reshape(16, 512).astype(np.float64)
    np.testing.assert_allclose(y, x.astype(np.float64) @ wd.T, rtol=1e-6, atol=1e-6)


def test_exp64_accuracy():
    """The shared binary64 exp (Cody-Waite + Taylor) is within 2 ulp of
    numpy's exp over the softmax / SiLU input range."""
    xs = np.concatenate([np.linspace(-740, 700, 20001), np.random.default_rng(0).normal(0, 5, 20000),
                         [0.0, -0.0, 1e-300, -1e-300, 0.5 * np.log(2), -0.5 * np.log(2)]])
    got = np.array([O.lib().or_exp64(float(v)) for v in xs])
    ref = np.exp(xs)
    ok = np.abs(got - ref) <= 2 * np.spacing(ref)
    assert ok.all(), xs[~ok][:5]
    assert O.lib().or_exp64(-800.0) == 0.0 and O.lib().or_exp64(800.0) == np.inf


def test_tensor_seed_convention_matches_product():
    """The oracle's per-tensor seed convention equals the product's
    (ferrite_b200.tensor_seed, used by fb_model_synth)."""
    import ferrite_b200 as fb
    for layer in (-1, 0, 5, 35):
        for name in O.KIND_ID:
            assert O.tensor_seed(99, layer, name) == fb.tensor_seed(99, layer, name)
