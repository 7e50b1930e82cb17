"""The skewed-routing stress config: the recorded bias constant gives the hottest expert about 10x
the mean load at T = 131072 (tests/golden/zipf_skew.json, made by moe_cases.calibrate_zipf_c), and some experts no
token at small T."""
import json

from moe_cases import ZIPF_FIXTURE, route_load_ratio, zipf_c


def test_recorded_zipf_constant_gives_ten_times_the_mean_load():
    c = zipf_c()
    ratio, _ = route_load_ratio(c, T=131072)
    assert 9.5 <= ratio <= 10.5
    assert route_load_ratio(c, T=16)[1] > 0          # empty experts at the tiny-group size
    d = json.load(open(ZIPF_FIXTURE))
    assert abs(d["measured_max_over_mean"] - ratio) < 1e-3
