"""tests/cases.py reproduces the reference's test matrices (qrbench/gen.py) bit for bit: fingerprints recorded from
the reference's own generator by tests/golden/make_golden.py."""
import json
from pathlib import Path

import pytest

from tests import cases

FIX = json.loads((Path(__file__).resolve().parent / "golden" / "reference_fixtures.json").read_text())


@pytest.mark.parametrize("shape", ["768x512", "3584x256"])
def test_generator_matches_reference(shape):
    K, r = map(int, shape.split("x"))
    n = 0
    for key, fp in FIX["gen_fingerprints"].items():
        if not key.startswith(shape + "/"):
            continue
        name = key.split("/")[1]
        assert cases.fingerprint(cases.make_case(K, r, name, 0)) == fp, key
        n += 1
    assert n == len(cases.case_names())


def test_baseline_configs_shapes_and_structure():
    import torch
    X0 = cases.cfg0()
    assert X0.shape == (768, 512) and X0.dtype == torch.float32
    s = torch.linalg.svdvals(X0.double())
    assert abs(float(s[0]) / 8 - 1) < 1e-5 and abs(float(s[0] / s[-1]) / 1e6 - 1) < 1e-3
    X3 = cases.cfg3_matrix(0, K=512, r=256)
    s3 = torch.linalg.svdvals(X3.double())
    assert float(s3[191] / s3[0]) > 1e-11 and float(s3[192] / s3[0]) < 1e-6    # rank 192 up to fp32 rounding
    Xa, Xb = cases.cfg2(1024, "base83"), cases.cfg2(1024, "scale_p83")
    assert torch.equal(Xa * 2.0 ** 83, Xb)      # exact power-of-2 scaling
