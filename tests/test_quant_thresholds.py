"""The device quantiser decides e2m1 codes without dividing: it compares |x| with per-block float thresholds
derived exactly from the scale (reax_engine_b200/csrc/common.cuh, e2m1_thresholds). This restates that derivation
in numpy and checks it against the reference's rule -- code of fl(x / sf) with engine/fp4.py's midpoint ties --
on values placed on and around every decision point."""
import numpy as np

from oracle import moe_oracle as O

C = np.array([0.25 + 2.0 ** -26, 0.75 - 2.0 ** -25, 1.25 + 2.0 ** -24, 1.75 - 2.0 ** -24,
              2.5 + 2.0 ** -23, 3.5 - 2.0 ** -23, 5.0 + 2.0 ** -22], dtype=np.float64)


def rd_f32(p):
    f = p.astype(np.float32)
    return np.where(f.astype(np.float64) > p, np.nextafter(f, np.float32(-np.inf)), f).astype(np.float32)


def thresholds(sf):
    P = C[None, :] * np.asarray(sf, np.float64)[:, None]          # exact in fp64 (<= 49 significant bits)
    f = rd_f32(P)
    nonstrict = (np.arange(7) % 2 == 1)[None, :]
    exact = f.astype(np.float64) == P
    return np.where(nonstrict & exact, np.nextafter(f, np.float32(0)), f).astype(np.float32)


def zero_threshold(sf):
    """RD(sf * 2^-150): |x| above it <=> fl(x / sf) does not underflow to 0 (the device's sign condition)."""
    z = np.asarray(sf, np.float64) * 2.0 ** -150
    return rd_f32(z)


def codes_by_threshold(x, sf):
    T = thresholds(sf)
    a = np.abs(x)[:, None]
    idx = (a > T).sum(axis=1).astype(np.uint8)
    return idx | (((x < 0) & (np.abs(x) > zero_threshold(sf))).astype(np.uint8) << 3)


def test_threshold_codes_equal_division_codes():
    rng = np.random.default_rng(0)
    n = 400000
    g = (rng.random(n).astype(np.float32) * np.float32(0.01) + np.float32(1e-4)).astype(np.float32)
    s8 = rng.integers(1, 126, n).astype(np.uint8)
    sf = np.maximum(O.e4m3_decode(s8) * g, np.float32(1e-30)).astype(np.float32)
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    m = mids[rng.integers(0, 7, n)]
    base = (m * sf).astype(np.float32)
    # x on the midpoint product and a few ulps either side (in fp32 and on the bf16 grid), random signs
    ulps = rng.integers(-3, 4, n).astype(np.int32)
    x = (base.view(np.int32) + ulps).view(np.float32)
    xb = O.bf16_round(x)
    xr = (rng.standard_normal(n).astype(np.float32) * sf * np.float32(3)).astype(np.float32)
    tiny = rng.integers(1, 1 << 16, n).astype(np.uint32).view(np.float32)      # fp32 denormals
    for xs in (x, xb, xr, -x, -xb, np.zeros(n, np.float32), -np.zeros(n, np.float32), -tiny):
        with np.errstate(under="ignore"):
            ref = O.e2m1_codes(np.clip((xs / sf).astype(np.float32), -6, 6))
        assert np.array_equal(codes_by_threshold(xs, sf), ref)


def codes_bf16_search(xb, sf):
    """The bf16x2 device path (quant_block16_bf16): thresholds truncated to bf16, a 3-level binary search on |x|,
    sign = x < 0 and |x| above the truncated zero threshold."""
    T = thresholds(sf)
    Tb = (T.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)
    a = np.abs(xb)
    b2 = a > Tb[:, 3]
    b1 = a > np.where(b2, Tb[:, 5], Tb[:, 1])
    t0 = np.where(b2, np.where(b1, Tb[:, 6], Tb[:, 4]), np.where(b1, Tb[:, 2], Tb[:, 0]))
    b0 = a > t0
    idx = (4 * b2 + 2 * b1 + b0).astype(np.uint8)
    zb = (zero_threshold(sf).view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)
    return idx | (((xb < 0) & (a > zb)).astype(np.uint8) << 3)


def test_bf16_binary_search_equals_division_codes():
    rng = np.random.default_rng(1)
    n = 400000
    g = (rng.random(n).astype(np.float32) * np.float32(0.01) + np.float32(1e-4)).astype(np.float32)
    s8 = rng.integers(1, 126, n).astype(np.uint8)
    sf = np.maximum(O.e4m3_decode(s8) * g, np.float32(1e-30)).astype(np.float32)
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    base = (mids[rng.integers(0, 7, n)] * sf).astype(np.float32)
    # bf16 values on and around every decision point (steps of one bf16 ulp), random values, signed zeros
    near = O.bf16_round(base)
    steps = rng.integers(-3, 4, n).astype(np.int32)
    xb = (((near.view(np.uint32) >> 16).astype(np.int32) + steps).astype(np.uint32) << 16).view(np.float32)
    xr = O.bf16_round((rng.standard_normal(n).astype(np.float32) * sf * np.float32(3)).astype(np.float32))
    for xs in (xb, -xb, xr, np.zeros(n, np.float32), -np.zeros(n, np.float32)):
        ref = O.e2m1_codes(np.clip((xs / sf).astype(np.float32), -6, 6))
        assert np.array_equal(codes_bf16_search(xs, sf), ref)


def test_bf16_binary_search_exhaustive_for_some_scales():
    """Every finite bf16 value of either sign against a handful of block scales, including the 1e-30 floor and
    scales large enough that the quotients of tiny values underflow to -0."""
    xb = (np.arange(0, 0x7F80, dtype=np.uint32) << 16).view(np.float32)
    for sfv in (1e-30, 3.0e-7, 0.0123, 0.5, 1.0, 7.25, 448.0 * 0.75, 1.5e6):
        sf = np.full(xb.shape[0], np.float32(sfv), np.float32)
        with np.errstate(under="ignore", over="ignore"):
            ref = O.e2m1_codes(np.clip((xb / sf).astype(np.float32), -6, 6))
            refn = O.e2m1_codes(np.clip((-xb / sf).astype(np.float32), -6, 6))
        assert np.array_equal(codes_bf16_search(xb, sf), ref)
        assert np.array_equal(codes_bf16_search(-xb, sf), refn)
