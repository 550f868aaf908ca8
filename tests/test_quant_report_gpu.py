"""The quantisation-accuracy report runs every format on one shape.  It
measures quantisation error (each format against the unquantised 16-bit
layer), so the bars here are on cosine similarity of the whole output and on
identical routing; the per-format parity bars (output vs an f32 reference of
the same quantised operands) are in the format's own tests."""
import pytest

from sparsemoe_b200.quant_report import report

pytestmark = pytest.mark.gpu

MIN_COSINE = {"int8_channel_token": 0.999, "fp8_e4m3_block": 0.995, "int4_g128": 0.98, "nvfp4_g16": 0.98}


def test_quant_report_small(gpu):
    rows = report(tokens=512, d=1024, f=512, experts=8, topk=2)
    assert len(rows) == 5
    for r in rows:
        assert r["routing_identical"], r
        assert r["cosine"] > MIN_COSINE.get(r["format"], 0.99), r
