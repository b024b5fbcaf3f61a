"""The CPU oracle against golden vectors produced by the reference's own
compiled kernel on a B200 (tests/golden/make_kernel_golden.py).

The oracle restates the kernel with the reference's contractions and double
requantisation but calls the host libm for expf / logf / powf, which can
differ from CUDA's by an ulp.  m involves none of them: m scales and codes
must be identical.  A one-ulp difference in log v moves v_min by one ulp,
scale_v = (max - min) / L by two log-ulps over L, and a v code by the number
of code steps two log-ulps span (zero or one at 4/8 bits, more at 16/32
bits); the tolerances below are exactly those bounds.  Parameters agree
within 1e-6 relative of max |p|.  The GPU kernel is held to bit-exactness against the
same vectors in tests/test_gpu_golden.py.
"""
import os

import numpy as np
import pytest

from oracle import oracle

GOLD = os.path.join(os.path.dirname(__file__), "golden", "kernel_golden.npz")
HP = (0.9, 0.999, 1e-3, 0.01, 1e-8)
LAYOUTS = ["packed4", "s8u8", "s16u16", "s32u32"]


def cases():
    g = np.load(GOLD)
    return sorted({k.split("/")[0] for k in g.files})


def ulp_diff(a, b):
    ai = a.view(np.int32).astype(np.int64)
    bi = b.view(np.int32).astype(np.int64)
    return np.abs(ai - bi)


@pytest.mark.parametrize("case", cases())
def test_oracle_matches_reference_kernel(case):
    g = np.load(GOLD)
    lay, bits, n, block = (int(x) for x in g[f"{case}/meta"])
    st = {k: g[f"{case}/in_{k}"].copy() for k in ("p", "m", "v", "sm", "sv", "vmin")}
    for s, grad in enumerate(g[f"{case}/grads"], start=1):
        oracle.step(st["p"], grad.astype(np.float32), lay, st["m"], st["v"] if st["v"].size else None,
                    st["sm"], st["sv"], st["vmin"], block, *HP, s, bits, bits)
    ref = {k: g[f"{case}/out_{k}"] for k in ("p", "m", "v", "sm", "sv", "vmin")}
    # m involves no transcendental: its scales and codes are exact.
    np.testing.assert_array_equal(st["sm"].view(np.int32), ref["sm"].view(np.int32))
    if LAYOUTS[lay] == "packed4":
        np.testing.assert_array_equal(st["m"] & 15, ref["m"] & 15)
    else:
        np.testing.assert_array_equal(st["m"], ref["m"])
    # log v: host logf vs CUDA logf differ by at most one ulp.
    assert ulp_diff(st["vmin"], ref["vmin"]).max() <= 1
    lv = float(2 ** bits - 1)
    lvmax = np.abs(ref["vmin"]) + ref["sv"] * lv                 # |log v| bound per block
    log_ulp = np.spacing(np.maximum(np.abs(ref["vmin"]), lvmax).astype(np.float32))
    tol_sv = 2 * log_ulp / lv + 2 * np.spacing(ref["sv"])
    assert (np.abs(st["sv"] - ref["sv"]) <= tol_sv).all()
    # a v code moves by at most the code width of two log ulps, plus one step
    qo = (st["m"] >> 4 if LAYOUTS[lay] == "packed4" else st["v"]).astype(np.int64)
    qr = (ref["m"] >> 4 if LAYOUTS[lay] == "packed4" else ref["v"]).astype(np.int64)
    blk = np.arange(n) // block
    bound = 1 + np.ceil(4 * log_ulp[blk] / ref["sv"][blk])
    assert (np.abs(qo - qr) <= bound).all()
    if bits <= 8:
        assert (qo != qr).mean() <= 2e-3
    assert np.abs(st["p"] - ref["p"]).max() <= 1e-6 * np.abs(ref["p"]).max()


def test_golden_file_covers_layouts_and_odd_blocks():
    g = np.load(GOLD)
    metas = [g[f"{c}/meta"] for c in cases()]
    assert {int(m[0]) for m in metas} == {0, 1, 2, 3}
    assert any(int(m[3]) & (int(m[3]) - 1) for m in metas)       # a non-power-of-two block
    assert any(int(m[2]) % int(m[3]) for m in metas)             # a partial tail block
