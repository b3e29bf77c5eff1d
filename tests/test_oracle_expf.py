"""The router's exp: glibc's expf (Rust's f32::exp, called by routed_moe at
har/crates/har-demo/src/bin/har-native-qwen35moe.rs:1176) restated as
Nagy's table-driven method, checked against the host's expf bit for bit.

The GPU router computes the same steps (expf_ref in the library), so its
routing weights are bit-exact against the reference's arithmetic; these CPU
tests pin the restatement itself: its table against 2^(i/32) rounded to
nearest double, and its results against glibc on every float of the router's
domain (logit - max in [-104, 0]) and of the non-overflowing positive range."""
import struct
import threading

import numpy as np
import pytest

import haro


def _bits(f: float) -> int:
    return struct.unpack("<I", struct.pack("<f", f))[0]


def test_exp2_table_is_correctly_rounded():
    mpmath = pytest.importorskip("mpmath")
    mpmath.mp.prec = 200
    for i, b in enumerate(haro.exp2_table()):
        want = struct.unpack("<Q", struct.pack("<d", float(mpmath.power(2, mpmath.mpf(i) / 32))))[0]
        assert b == want, i


def _exhaustive(lo: int, hi: int, parts: int = 8):
    """Mismatch count over bit patterns lo..hi, split across threads."""
    step = (hi - lo + parts) // parts
    res = [None] * parts

    def run(j):
        a = lo + j * step
        b = min(hi, a + step - 1)
        res[j] = haro.expf_mismatches(a, b) if a <= b else (0, 0)

    th = [threading.Thread(target=run, args=(j,)) for j in range(parts)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    return sum(r[0] for r in res), [r[1] for r in res if r[0]]


def test_restated_expf_equals_glibc_on_router_domain():
    # every float in [-104, -0]: bit patterns 0x80000000 .. bits(-104)
    n, first = _exhaustive(0x80000000, _bits(-104.0))
    assert n == 0, f"{n} mismatches, first at {first}"


def test_restated_expf_equals_glibc_on_positive_range():
    n, first = _exhaustive(0, _bits(88.72))
    assert n == 0, f"{n} mismatches, first at {first}"


def test_router_weights_restated_equal_glibc():
    lg = haro.normal_f32(31, 0, 256 * 512).reshape(256, 512) * np.float32(4.0)
    i0, w0 = haro.route_topk(lg, 10, exp_mode=0)
    i2, w2 = haro.route_topk(lg, 10, exp_mode=2)
    assert np.array_equal(i0, i2)
    assert np.array_equal(w0.view(np.uint32), w2.view(np.uint32))


def test_special_values():
    assert haro.expf_restated(0.0) == 1.0
    assert haro.expf_restated(-200.0) == 0.0
    assert haro.expf_restated(float("-inf")) == 0.0
    assert haro.expf_restated(100.0) == float("inf")
