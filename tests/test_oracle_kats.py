"""The oracle against the reference's own known-answer tests (CPU only).

Each case cites the reference test it transcribes (tests/golden/reference_kats.json).
"""
import numpy as np
import pytest

import haro
from _common import kats

K = kats()


@pytest.mark.parametrize("b0,b1,expected", K["f16_to_f32"]["cases"])
def test_f16_conversion_is_exact(b0, b1, expected):
    # har/crates/har-serve/src/q4k.rs:235-244 (both converters must agree)
    v = haro.f16_to_f32(b0, b1)
    assert np.float32(v) == np.float32(expected)
    assert np.signbit(v) == np.signbit(expected)
    assert haro.half_to_f32(b0 | (b1 << 8)) == np.float32(expected)


def test_f16_converters_agree_on_all_bit_patterns():
    # q4k.rs:22-50 (arithmetic) and har-native-qwen3.rs:116-136 (bit construction)
    for bits in range(0, 1 << 16):
        a = haro.f16_to_f32(bits & 0xFF, bits >> 8)
        b = haro.half_to_f32(bits)
        if np.isnan(a):
            assert np.isnan(b)
        else:
            assert np.float32(a).tobytes() == np.float32(b).tobytes(), hex(bits)


def test_dequant_matches_synthetic_gguf_fixture():
    # har/crates/har-serve/src/q4k.rs:226-258: d = 1.0, scales and codes zero -> dot 0
    block = np.zeros(144, np.uint8)
    block[1] = 0x3C
    x = haro.lcg_values(256, 17)
    dot = np.float32(0.0)
    for i in range(256):
        dot = np.float32(dot + np.float32(haro.q4k_dequant(block, i)) * x[i])
    assert abs(float(dot) - K["zero_scale_block_dot"]["expected"]) < K["zero_scale_block_dot"]["abs_tol"]
    assert abs(haro.q4k_dot(block, x)) < 1e-6


def test_lcg_values_regression():
    assert list(map(float, haro.lcg_values(8, 17))) == K["lcg_values"]["first8_seed17"]
    v = haro.lcg_values(10000, 5)
    assert v.min() >= -0.5 and v.max() < 0.5


def test_q4_zero_block_decodes_to_zero():
    # har/crates/har-demo/src/bin/har-native-qwen3.rs:1533-1540
    out = haro.decode_q4k_block(np.zeros(144, np.uint8))
    assert np.all(out == 0.0)


def smoke_block():
    kat = K["vulkan_smoke_q4k_gemv"]["block"]
    block = np.zeros(144, np.uint8)
    block[1] = kat["byte1"]
    block[4:16] = kat["bytes_4_16"]
    block[16:] = kat["bytes_16_144"]
    return block


def test_vulkan_smoke_known_answer():
    # har/crates/har-vulkan/src/bin/smoke.rs:96-160: expected 256.0
    block = smoke_block()
    x = np.ones(256, np.float32)
    exp = K["vulkan_smoke_q4k_gemv"]["expected"]
    assert abs(float(haro.q4k_matvec(block, 1, 256, x)[0]) - exp) < 1e-4
    assert abs(haro.q4k_dot(block, x) - exp) < 1e-4


def test_top_k_tie_order_is_deterministic():
    # har-native-qwen35moe.rs:1508-1519: equal probabilities -> lower index first
    logits = np.zeros((1, 3), np.float32)
    ids, w = haro.route_topk(logits, 3)
    assert list(ids[0]) == K["top_k_tie_order"]["expected_order"]
    assert np.allclose(w, 1.0 / 3.0)


def test_router_topk_weights_sum_to_one():
    # har/crates/har-serve/src/moe.rs:348-356 (tolerance 1e-5)
    logits = haro.normal_f32(3, 0, 16 * 512).reshape(16, 512)
    ids, w = haro.route_topk(logits, 10)
    assert np.all(np.abs(w.sum(axis=1) - 1.0) < K["router_topk_weights_sum_to_one"]["abs_tol"])
    for t in range(16):
        assert len(set(ids[t])) == 10
        p = np.exp(logits[t].astype(np.float64) - logits[t].max())
        assert list(ids[t]) == list(np.argsort(-p, kind="stable")[:10])


def test_q4k_row_geometry():
    # har/crates/har-package-slice/src/tests.rs:48,480: 5120 columns -> 2880 B rows
    kat = K["q4k_row_bytes"]
    assert kat["columns"] // 256 * 144 == kat["expected_row_bytes"]
    row = haro.gen_q4k(1, 1, kat["columns"])
    assert row.shape == (1, kat["expected_row_bytes"])


def test_serving_and_expert_orders_agree():
    # q4k.rs:170-188 (one accumulator over all values) vs q4k_dot's per-block
    # sums (har-native-qwen3.rs:149-172): same dequantised values, different
    # f32 summation order -> within accumulation-order tolerance.
    w = haro.gen_q4k(9, 32, 2048)
    x = haro.normal_f32(10, 0, 2048)
    a = haro.q4k_matvec(w, 32, 2048, x)
    b = np.array([haro.dot_quant_row(w[r], x) for r in range(32)], np.float32)
    assert np.max(np.abs(a - b)) / np.max(np.abs(a)) < 1e-5
