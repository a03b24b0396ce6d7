"""The CPU-vs-GPU demo report (tests/demo_report.py) on cuda:0: every program
runs through `sample_states`, its chains follow the oracle's trajectories and
the pooled statistics of both sides agree."""

from __future__ import annotations

import numpy as np
import pytest

import demo_report

pytestmark = pytest.mark.gpu


def test_demo_report_matches_oracle(cuda_device, capsys):
    results = demo_report.main(["--chains", "1024", "--profile"])
    out = capsys.readouterr().out
    assert "speedup" in out and "dispatch" in out
    assert len(results) == 4
    for r in results:
        # a chain leaves the oracle's trajectory only after a draw inside the 1e-5 band
        assert r.chains_matching >= 0.99, (r.name, r.chains_matching)
        assert r.timing, r.name
        for g, c in zip(r.gpu, r.cpu):
            assert g.shape == c.shape, r.name
            if np.issubdtype(g.dtype, np.floating):
                np.testing.assert_allclose(g.mean(), c.mean(), rtol=1e-3, atol=5e-3)
            else:
                assert abs(float(g.astype(float).mean()) - float(c.astype(float).mean())) < 1e-2, r.name
