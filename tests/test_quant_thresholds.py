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


def codes_by_threshold(x, sf):
    T = thresholds(sf)
    a = np.abs(x)[:, None]
    idx = (a > T).sum(axis=1).astype(np.uint8)
    return idx | ((x < 0).astype(np.uint8) << 3)


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
    for xs in (x, xb, xr, -x, -xb, np.zeros(n, np.float32), -np.zeros(n, np.float32)):
        ref = O.e2m1_codes(np.clip((xs / sf).astype(np.float32), -6, 6))
        assert np.array_equal(codes_by_threshold(xs, sf), ref)
