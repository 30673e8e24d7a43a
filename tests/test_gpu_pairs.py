"""The CTA-pair MXFP4 kernel (k_gemm_mxf4_pair: two adjacent column tiles
as one tcgen05 MMA of M = 256 on a cluster of two CTAs, opt-in with
HRB_CTA_PAIRS=1) gives the same bits as one CTA a tile (k_gemm_mxf4) on
every output, MXINT8 copy included: the same products, added in the same
order.  The one-CTA kernel is itself checked against the float64 product in
tests/test_gpu_fast.py and tests/test_gpu_large.py.  Each kernel runs in a
child process (tests/pairs_worker.py), since the choice is made once per
process."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

HERE = os.path.dirname(os.path.abspath(__file__))


def run_worker(out, pairs):
    env = dict(os.environ, HRB_CTA_PAIRS="1" if pairs else "0")
    r = subprocess.run([sys.executable, os.path.join(HERE, "pairs_worker.py"), str(out)],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]


def test_pair_kernel_bit_equal_to_one_cta_a_tile(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    pair, single = tmp_path / "pair", tmp_path / "single"
    pair.mkdir()
    single.mkdir()
    run_worker(pair, True)
    run_worker(single, False)
    names = sorted(os.listdir(pair))
    assert names == sorted(os.listdir(single)) and len(names) >= 10
    for name in names:
        a, b = np.load(pair / name), np.load(single / name)
        assert a.tobytes() == b.tobytes(), f"{name}: {int((a != b).sum())} elements differ"
