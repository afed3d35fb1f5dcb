"""The GEMV's weight stages and the decode attention's K / V tiles can be requested as
one 3-D / 4-D TMA box each or as several 2-D boxes; both forms must put the same bytes
at the same shared-memory addresses, so every output is bit-identical.  The form is
chosen once per process (HM_GEMV_BOX, HM_ATTN_BOX), so each runs in a child process
(tests/box_ab_child.py) and the outputs are compared here."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent


def _run(tmp_path, box):
    env = dict(os.environ, HM_GEMV_BOX=str(box), HM_ATTN_BOX=str(box))
    f = tmp_path / f"box{box}.pt"
    r = subprocess.run([sys.executable, str(HERE / "box_ab_child.py"), str(f)], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return torch.load(f)


def test_one_box_per_stage_equals_2d_boxes(tmp_path):
    from estudiocanciones_b200 import build
    build.build()
    a, b = _run(tmp_path, 0), _run(tmp_path, 1)
    assert a.keys() == b.keys()
    assert int(a["errors"]) == 0 and int(b["errors"]) == 0
    # every shape here has K % 128 == 0, so the one-box form is taken whenever it is on
    assert (a.pop("forms") == 0).all() and (b.pop("forms") == 1).all()
    for k in a:
        assert torch.equal(a[k], b[k]), f"{k} differs between the box forms"
