"""Config: the reference's geometry validation and derived sizes (DS/runtime.py:19-96)."""
import importlib

import pytest

C = importlib.import_module("10_20_b200.config").Config


def test_defaults_and_derived_sizes():
    c = C()
    assert c.pages == 1024 and c.take == 512 and c.width == 37120
    assert c.ratio.numerator == 1 and c.ratio.denominator == 2
    # decode geometry of the benchmark: 128K context, a 40-page budget rounds to topk/64 = 32 minimum
    d = C(max_context=131072, heads=64, topk=2048, page_fraction=40 / 2048, window=64, max_requests=128)
    assert d.pages == 2048 and d.take == 40 and d.width == 6912
    cap = d.pages * d.max_requests
    expect = (cap * (8448 + 1056 + 256 + 32) + 64 * 68 * 8448 + 128 * 2048 * 4 + (32 << 20)
              + sum((8 << 20) + r * (6912 * 24 + 2048 * 64 + 32768) for r in (1, 4, 16, 64)))
    assert d.reservation == expect
    e = C(expand_output=True)
    assert e.reservation == C().reservation + 85 * (512 * 4 + 64) * 4


@pytest.mark.parametrize("kw", [dict(max_context=4095), dict(max_context=6000), dict(topk=0), dict(topk=2049),
                                dict(page_fraction=0), dict(heads=16), dict(score_mode="x"), dict(sink=32),
                                dict(window=4097), dict(q_buckets=()), dict(q_buckets=(2, 4)),
                                dict(q_buckets=(4, 1)), dict(budget_bytes=0), dict(max_requests=0)])
def test_invalid_geometry_rejected(kw):
    with pytest.raises(ValueError):
        C(**kw)
