"""The codec's SnakeBeta evaluates sin^2 with a Cody-Waite reduction modulo pi
followed by the __sinf intrinsic on [-pi/2, pi/2] (codec.cu, sin_sq).  This
test reads the reduction constants from that function and replays the
reduction in f32 (numpy, one rounding per operation; the device uses FMAs and
is at least as accurate), with the sine of the reduced argument perturbed by
the intrinsic's documented worst-case absolute error (2^-21.41 on [-pi, pi]),
and checks the bound the comment states against the f64 sine:
max |sin_sq(y) - sin(y)^2| < 1e-6 for |y| <= 3000, with the reduced argument
inside [-pi/2, pi/2]."""
import os
import re

import numpy as np

SRC = os.path.join(os.path.dirname(__file__), "..", "tts-rs_b200", "csrc", "codec.cu")


def sin_sq_constants():
    src = open(SRC).read()
    body = src[src.index("Q3T_DEV float sin_sq(float y) {"):]
    body = body[:body.index("\n}\n")]
    return [float(x) for x in re.findall(r"(-?\d+\.\d+(?:e-?\d+)?)f", body)]


def test_sin_sq_error_bound():
    c = [np.float32(x) for x in sin_sq_constants()]
    inv_pi, pa, pb, pc = c
    assert inv_pi == np.float32(1 / np.pi) and float(pa) == 3.140625
    assert abs(float(pa) + float(pb) + float(pc) - np.pi) < 1e-12
    y = np.linspace(-3000, 3000, 3_000_001, dtype=np.float32)
    k = np.rint(y * inv_pi).astype(np.float32)
    r = (y - k * pa).astype(np.float32)
    r = (r - k * pb).astype(np.float32)
    r = (r - k * pc).astype(np.float32)
    assert np.abs(r).max() <= np.pi / 2 + 1e-3
    ref = np.sin(y.astype(np.float64)) ** 2
    for e in (-(2.0 ** -21.41), 2.0 ** -21.41):  # the intrinsic's error bound, either sign
        sn = np.sin(r.astype(np.float64)) + e
        assert np.abs(sn * sn - ref).max() < 1e-6
