"""The oracle against the committed golden vectors, and oracle-internal
properties (CPU only)."""
import numpy as np

import haro
from _common import golden, rel_max

G = golden()


def test_gemv_golden():
    w, x = G["gemv_w"], G["gemv_x"]
    assert np.array_equal(haro.q4k_matvec(w, 64, 1024, x), G["gemv_y_serve"])
    y = np.array([haro.dot_quant_row(w[r], x) for r in range(64)], np.float32)
    assert np.array_equal(y, G["gemv_y_expert"])


def test_q8k_golden():
    xq = haro.q8k_quantize(G["gemv_x"].reshape(1, -1))
    assert np.array_equal(xq, G["gemv_xq"])
    assert np.array_equal(haro.q4k_gemv_q8k(G["gemv_w"], 64, 1024, xq), G["gemv_y_q8k"])


def test_route_golden():
    ids, w = haro.route_topk(G["route_logits"], 8)
    assert np.array_equal(ids, G["route_ids"]) and np.array_equal(w, G["route_w"])


def test_moe_golden():
    E, H, I, T, k = (int(v) for v in G["moe_dims"])
    y = haro.moe_ffn(G["moe_wg"], G["moe_wu"], G["moe_wd"], (G["moe_sg"], G["moe_su"], G["moe_sd"]),
                     G["moe_gi"], E, H, I, G["moe_x"], G["moe_ids"], G["moe_w"], threads=1)
    assert np.array_equal(y, G["moe_y"])
    # row-chunk threading (expert_matvec's scoped workers) must not change a bit
    y4 = haro.moe_ffn(G["moe_wg"], G["moe_wu"], G["moe_wd"], (G["moe_sg"], G["moe_su"], G["moe_sd"]),
                      G["moe_gi"], E, H, I, G["moe_x"], G["moe_ids"], G["moe_w"], threads=4)
    assert np.array_equal(y4, G["moe_y"])


def test_q8k_quantise_properties():
    x = np.concatenate([haro.normal_f32(5, 0, 256 * 7), np.zeros(256, np.float32)]).reshape(2, 1024)
    x[0, 5] = 1e-39  # subnormal input
    q = haro.q8k_quantize(x)
    for m in range(2):
        for b in range(4):
            blk = q[m, b * 292:(b + 1) * 292]
            d = blk[:4].view(np.float32)[0]
            qs = blk[4:260].view(np.int8).astype(np.int32)
            bs = blk[260:292].view(np.int16)
            v = x[m, 256 * b:256 * (b + 1)]
            amax = np.abs(v).max()
            assert d == np.float32(amax / np.float32(127.0))
            assert np.all(np.abs(qs) <= 127)
            assert np.array_equal(bs, qs.reshape(16, 16).sum(axis=1))
            if amax > 0:
                assert np.max(np.abs(qs * d - v)) <= 0.5001 * d + 1e-30
            else:
                assert np.all(qs == 0) and d == 0.0


def test_q4k_quantiser_roundtrip():
    x = haro.normal_f32(11, 0, 256 * 64, 0.0, 0.02).reshape(64, 256)
    q = haro.q4k_quantize(x)
    deq = np.stack([haro.decode_q4k_block(q[i]) for i in range(64)])
    err = np.sqrt(np.mean((deq - x) ** 2)) / np.std(x)
    assert err < 0.12  # 4-bit codes with 6-bit sub-block scales
    # every encoded block decodes identically through both reference decoders
    for i in range(8):
        assert np.array_equal(deq[i], np.array([haro.q4k_dequant(q[i], j) for j in range(256)], np.float32))


def test_group_by_expert_is_stable():
    ids, _ = haro.zipf_routing(3, 50, 64, 6)
    counts, offsets, order = haro.group_by_expert(ids, 64)
    flat = ids.reshape(-1)
    assert counts.sum() == flat.size and offsets[-1] == flat.size
    for e in range(64):
        members = order[offsets[e]:offsets[e + 1]]
        assert np.all(flat[members] == e)
        assert np.all(np.diff(members) > 0)  # position order (moe.rs:197-202)


def test_zipf_routing_shape():
    ids, w = haro.zipf_routing(1, 256, 512, 10)
    assert ids.shape == (256, 10)
    assert all(len(set(r)) == 10 for r in ids)
    assert np.all(np.abs(w.sum(1) - 1) < 1e-5)
    counts = np.bincount(ids.ravel(), minlength=512)
    assert counts.max() > 150  # heavy head: the hottest expert is in most tokens


def test_correctly_rounded_exp_mode_keeps_ids():
    lg = haro.normal_f32(21, 0, 64 * 512).reshape(64, 512)
    i0, w0 = haro.route_topk(lg, 10, exp_mode=0)
    i1, w1 = haro.route_topk(lg, 10, exp_mode=1)
    assert np.array_equal(i0, i1)
    assert rel_max(w1, w0) < 1e-6


def test_router_and_q6k_golden():
    """The router GEMV and Q6_K restatements against their frozen outputs
    (tests/golden/oracle_vectors_router_q6k.npz, written by make_golden.py)."""
    import os
    from _common import GOLDEN
    R = np.load(os.path.join(GOLDEN, "oracle_vectors_router_q6k.npz"))
    got = haro.router_logits(R["router_w"], R["router_x"])
    assert np.array_equal(got.view(np.uint32), R["router_logits"].view(np.uint32))
    y = haro.q6k_matvec(R["q6k_w"], 12, 768, R["q6k_x"])
    assert np.array_equal(y.view(np.uint32), R["q6k_y"].view(np.uint32))


def test_q6k_geometry_known_answer():
    """har-native-qwen3.rs:37 and har-model/src/lib.rs:609,626: Q6_K is GGML
    type 14, 210 bytes per 256 values — the oracle, the host layer and the
    GGUF type table agree."""
    import har_cuda
    from _common import kats
    k = kats()["q6k_geometry"]
    assert haro.Q6K_BLOCK_BYTES == k["block_bytes"] == har_cuda.Q6K_BLOCK_BYTES
    assert har_cuda.GGML_Q6_K == k["ggml_type"]
    assert har_cuda.BLOCK_BYTES[k["ggml_type"]] == k["block_bytes"]
