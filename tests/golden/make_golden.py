"""Writes the golden fixtures under tests/golden/.

1. reference_kats.json — known-answer values transcribed from the reference's
   own tests for this path (leoinfer/remora-lab; path:line of each source is
   stored beside the value).  The reference is Rust and cannot be built in
   this image, so its tests are read as text and their literals recorded.
2. oracle_vectors.npz — small seeded inputs and the C oracle's outputs (HAR's
   CPU arithmetic restated, oracle/har_oracle.c).  These pin the oracle
   against regressions and give the GPU tests fixed expected outputs.
3. oracle_vectors_router_q6k.npz — the same for the router GEMV
   (routed_moe's matvec(ffn_gate_inp)) and the Q6_K dot / matvec.

Run from the repository root:  python tests/golden/make_golden.py
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import haro  # noqa: E402

KATS = {
    "f16_to_f32": {
        "source": "har/crates/har-serve/src/q4k.rs:235-244",
        "cases": [  # (byte0, byte1, expected f32)
            [0x00, 0x3C, 1.0], [0x00, 0x00, 0.0], [0x00, 0x80, -0.0], [0x00, 0xBC, -1.0],
            [0x01, 0x3C, 1.0009766], [0x01, 0x00, 5.9604645e-8], [0x00, 0x03, 4.5776367e-5],
        ],
    },
    "zero_scale_block_dot": {
        "source": "har/crates/har-serve/src/q4k.rs:226-258",
        "block": {"d_bits": 0x3C00, "rest": 0},
        "input": "lcg_values(256, 17)",
        "expected": 0.0, "abs_tol": 1e-6,
    },
    "lcg_values": {
        "source": "har/crates/har-serve/src/q4k.rs:109-120",
        "note": "generator restated; first values recorded from the oracle for regression",
    },
    "zero_block_decodes_to_zero": {
        "source": "har/crates/har-demo/src/bin/har-native-qwen3.rs:1533-1540",
        "expected": 0.0,
    },
    "vulkan_smoke_q4k_gemv": {
        "source": "har/crates/har-vulkan/src/bin/smoke.rs:96-160",
        "block": {"byte1": 0x3C, "bytes_4_16": 1, "bytes_16_144": 0x11},
        "input": "256 x 1.0", "expected": 256.0, "abs_tol": 1e-4,
    },
    "top_k_tie_order": {
        "source": "har/crates/har-demo/src/bin/har-native-qwen35moe.rs:1508-1519",
        "probabilities": [1.0, 1.0, 1.0], "expected_order": [0, 1, 2],
    },
    "router_topk_weights_sum_to_one": {
        "source": "har/crates/har-serve/src/moe.rs:348-356", "abs_tol": 1e-5,
    },
    "q4k_row_bytes": {
        "source": "har/crates/har-package-slice/src/tests.rs:48,480",
        "columns": 5120, "expected_row_bytes": 2880,
    },
    "engine_verdict": {
        "source": "har/crates/har-execution/src/lib.rs:185-195,285-299",
        "normalized_rms_max": 5e-5, "max_abs_max": 5e-3,
    },
    "smoke_tolerance": {
        "source": "har/crates/har-serve/src/bin/har-serve-vulkan-batched-smoke.rs:63-76",
        "max_abs_logit_error": 1e-4,
    },
    "q6k_geometry": {
        "source": "har/crates/har-demo/src/bin/har-native-qwen3.rs:37; har/crates/har-model/src/lib.rs:609,626",
        "ggml_type": 14, "block_values": 256, "block_bytes": 210,
    },
    "router_constants": {
        "source": "har/crates/har-demo/src/bin/har-native-qwen35moe.rs:45-46",
        "TOP_K": 8, "ROUTER_EPS": 1e-9,
    },
}


def main():
    kats = dict(KATS)
    kats["lcg_values"]["first8_seed17"] = [float(v) for v in haro.lcg_values(8, 17)]
    with open(os.path.join(HERE, "reference_kats.json"), "w") as f:
        json.dump(kats, f, indent=1)

    rng_seed = 20261201
    # Q4_K GEMV: 64 rows x 1024 (4 blocks per row)
    w = haro.gen_q4k(rng_seed, 64, 1024)
    x = haro.normal_f32(rng_seed + 1, 0, 1024)
    y_serve = haro.q4k_matvec(w, 64, 1024, x)            # q4k.rs:170-188 order
    y_expert = np.array([haro.dot_quant_row(w[r], x) for r in range(64)], np.float32)
    xq = haro.q8k_quantize(x.reshape(1, -1))
    y_q8k = haro.q4k_gemv_q8k(w, 64, 1024, xq)
    # router: 6 tokens over 64 experts, k = 8
    logits = haro.normal_f32(rng_seed + 2, 0, 6 * 64).reshape(6, 64)
    ids, wts = haro.route_topk(logits, 8)
    # a small MoE layer: E=4, H=256, I=256, k=2, T=3, shared expert + gate row
    E, H, I, T, k = 4, 256, 256, 3, 2
    wg = haro.gen_q4k(rng_seed + 3, E * I, H)
    wu = haro.gen_q4k(rng_seed + 4, E * I, H)
    wd = haro.gen_q4k(rng_seed + 5, E * H, I)
    sg = haro.gen_q4k(rng_seed + 6, I, H)
    su = haro.gen_q4k(rng_seed + 7, I, H)
    sd = haro.gen_q4k(rng_seed + 8, H, I)
    gi = haro.normal_f32(rng_seed + 9, 0, H, 0.0, 0.02)
    xm = haro.normal_f32(rng_seed + 10, 0, T * H).reshape(T, H)
    ml = haro.normal_f32(rng_seed + 11, 0, T * E).reshape(T, E)
    mids, mw = haro.route_topk(ml, k)
    ym = haro.moe_ffn(wg, wu, wd, (sg, su, sd), gi, E, H, I, xm, mids, mw, threads=1)
    np.savez_compressed(os.path.join(HERE, "oracle_vectors.npz"),
                        gemv_w=w, gemv_x=x, gemv_y_serve=y_serve, gemv_y_expert=y_expert,
                        gemv_xq=xq, gemv_y_q8k=y_q8k,
                        route_logits=logits, route_ids=ids, route_w=wts,
                        moe_wg=wg, moe_wu=wu, moe_wd=wd, moe_sg=sg, moe_su=su, moe_sd=sd,
                        moe_gi=gi, moe_x=xm, moe_ids=mids, moe_w=mw, moe_y=ym,
                        moe_dims=np.array([E, H, I, T, k], np.int64))
    # router GEMV: 5 tokens, 48 experts, H = 320 (not a multiple of 64); Q6_K:
    # 12 rows x 768 values, 2 tokens
    rw = haro.normal_f32(rng_seed + 12, 0, 48 * 320, 0.0, 0.02).reshape(48, 320)
    rx = haro.normal_f32(rng_seed + 13, 0, 5 * 320).reshape(5, 320)
    rl = haro.router_logits(rw, rx)
    q6 = haro.random_q6k(rng_seed + 14, 12, 768)
    q6x = haro.normal_f32(rng_seed + 15, 0, 2 * 768).reshape(2, 768)
    q6y = haro.q6k_matvec(q6, 12, 768, q6x)
    np.savez_compressed(os.path.join(HERE, "oracle_vectors_router_q6k.npz"),
                        router_w=rw, router_x=rx, router_logits=rl,
                        q6k_w=q6, q6k_x=q6x, q6k_y=q6y)
    print("wrote", HERE)


if __name__ == "__main__":
    main()
