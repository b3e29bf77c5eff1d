"""ctypes binding of the CPU oracle (oracle/har_oracle.c).

TEST INFRASTRUCTURE ONLY: tests/, ``__graft_entry__.smoke()`` and bench.py's
CPU-baseline leg use this module as the checker.  The product path
(``har_cuda``) never imports it.  Each wrapper names the reference function
the C code restates (paths relative to the leoinfer/remora-lab root).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libhar_oracle.so")

QK_K = 256
Q4K_BLOCK_BYTES = 144
Q8K_BLOCK_BYTES = 292
ROUTER_EPS = 1.0e-9

_lib = None

_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64 = C.c_int64


def build() -> str:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    L = C.CDLL(LIB_PATH)
    sig = {
        "haro_f16_to_f32": (C.c_float, [C.c_uint8, C.c_uint8]),
        "haro_half_to_f32": (C.c_float, [C.c_uint16]),
        "haro_f32_to_f16_rne": (C.c_uint16, [C.c_float]),
        "haro_scale_at": (C.c_uint32, [_u8p, C.c_int]),
        "haro_min_at": (C.c_uint32, [_u8p, C.c_int]),
        "haro_q4k_dequant": (C.c_float, [_u8p, C.c_int]),
        "haro_decode_q4k_block": (None, [_u8p, _f32p]),
        "haro_q4k_matvec": (None, [_u8p, _i64, _i64, _f32p, _f32p]),
        "haro_q4k_dot": (C.c_float, [_u8p, _f32p]),
        "haro_dot_quant_row": (C.c_float, [_u8p, _f32p, _i64]),
        "haro_expert_matvec": (None, [_u8p, _i64, _i64, _i64, _i64, _f32p, _f32p, C.c_int]),
        "haro_silu": (C.c_float, [C.c_float]),
        "haro_sigmoid": (C.c_float, [C.c_float]),
        "haro_route_topk": (None, [_f32p, C.c_int, C.c_int, _i32p, _f32p]),
        "haro_router_logits": (None, [_f32p, _i64, _i64, _f32p, _f32p]),
        "haro_q6k_dot": (C.c_float, [_u8p, _f32p]),
        "haro_q6k_matvec": (None, [_u8p, _i64, _i64, _f32p, _f32p]),
        "haro_q3k_scale": (C.c_int, [_u8p, C.c_int]),
        "haro_q3k_dequant_block": (None, [_u8p, _f32p]),
        "haro_q3k_dot": (C.c_float, [_u8p, _f32p]),
        "haro_q3k_matvec": (None, [_u8p, _i64, _i64, _f32p, _f32p]),
        "haro_group_by_expert": (None, [_i64, C.c_int, C.c_int, _i32p, _i32p, _i32p, _i32p]),
        "haro_q8k_quantize": (None, [_f32p, _i64, _u8p]),
        "haro_q8k_dot_row": (C.c_float, [_u8p, _u8p, _i64]),
        "haro_q4k_gemv_q8k": (None, [_u8p, _i64, _i64, _u8p, _f32p]),
        "haro_q4k_quantize_row": (None, [_f32p, _i64, _u8p]),
        "haro_lcg_values": (None, [_i64, C.c_uint64, _f32p]),
        "haro_normal_f32": (None, [C.c_uint64, _i64, _i64, C.c_float, C.c_float, _f32p]),
        "haro_gen_q4k_rows": (None, [C.c_uint64, _i64, _i64, _i64, C.c_float, C.c_float, _u8p]),
        "haro_zipf_routing": (None, [C.c_uint64, _i64, C.c_int, C.c_int, C.c_double, _i32p, _f32p]),
        "haro_online_cpus": (C.c_int, []),
        "haro_set_exp_mode": (None, [C.c_int]),
        "haro_expf_restated": (C.c_float, [C.c_float]),
        "haro_exp2_table": (None, [C.POINTER(C.c_uint64)]),
        "haro_expf_mismatches": (C.c_uint64, [C.c_uint32, C.c_uint32, C.POINTER(C.c_uint32)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    vp = C.c_void_p
    for name in ("haro_moe_ffn", "haro_moe_ffn_q8k"):
        fn = getattr(L, name)
        fn.restype = None
        fn.argtypes = [vp, vp, vp, vp, vp, vp, vp, _i64, _i64, _i64, _i64, C.c_int,
                       vp, vp, vp, C.c_int, vp, C.c_int]
    _lib = L
    return L


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# ---- a1-a5 -----------------------------------------------------------------

def f16_to_f32(b0: int, b1: int) -> float:
    """har/crates/har-serve/src/q4k.rs:22-50"""
    return lib().haro_f16_to_f32(b0, b1)


def half_to_f32(v: int) -> float:
    """har/crates/har-demo/src/bin/har-native-qwen3.rs:116-136"""
    return lib().haro_half_to_f32(v)


def q4k_dequant(block: np.ndarray, index: int) -> float:
    """har/crates/har-serve/src/q4k.rs:77-89"""
    return lib().haro_q4k_dequant(np.ascontiguousarray(block, np.uint8), index)


def decode_q4k_block(block: np.ndarray) -> np.ndarray:
    """har/crates/har-demo/src/bin/har-native-qwen3.rs:1067-1093"""
    out = np.empty(QK_K, np.float32)
    lib().haro_decode_q4k_block(np.ascontiguousarray(block, np.uint8), out)
    return out


def q4k_matvec(w: np.ndarray, rows: int, dim: int, x: np.ndarray) -> np.ndarray:
    """har/crates/har-serve/src/q4k.rs:170-188 (Q4KModel::matvec)"""
    out = np.empty(rows, np.float32)
    lib().haro_q4k_matvec(np.ascontiguousarray(w, np.uint8).reshape(-1), rows, dim,
                          np.ascontiguousarray(x, np.float32), out)
    return out


def q4k_dot(block: np.ndarray, x: np.ndarray) -> float:
    """har/crates/har-demo/src/bin/har-native-qwen3.rs:149-172"""
    return lib().haro_q4k_dot(np.ascontiguousarray(block, np.uint8),
                              np.ascontiguousarray(x, np.float32))


def dot_quant_row(row: np.ndarray, x: np.ndarray) -> float:
    """har/crates/har-demo/src/bin/har-native-qwen3.rs:207-232"""
    x = np.ascontiguousarray(x, np.float32)
    return lib().haro_dot_quant_row(np.ascontiguousarray(row, np.uint8), x, x.size)


def expert_matvec(tensor: np.ndarray, E: int, N: int, K: int, expert: int,
                  x: np.ndarray, threads: int = 0) -> np.ndarray:
    """har/crates/har-demo/src/bin/har-native-qwen35moe.rs:626-689"""
    y = np.empty(N, np.float32)
    lib().haro_expert_matvec(np.ascontiguousarray(tensor, np.uint8).reshape(-1), E, N, K,
                             expert, np.ascontiguousarray(x, np.float32), y, threads)
    return y


def silu(v: float) -> float:
    return lib().haro_silu(v)


def sigmoid(v: float) -> float:
    return lib().haro_sigmoid(v)


def route_topk(logits: np.ndarray, k: int, exp_mode: int = 0):
    """har/crates/har-demo/src/bin/har-native-qwen35moe.rs:1167-1204, per row.

    exp_mode 0 uses glibc's expf (the reference's f32::exp); 2 its
    restatement (haro_expf_restated, the steps the GPU router computes; equal
    to mode 0 bit for bit); 1 the correctly rounded exp (differs from glibc's
    on ~1 in 11,500 inputs)."""
    lib().haro_set_exp_mode(exp_mode)
    logits = np.ascontiguousarray(logits, np.float32)
    T, E = logits.shape
    ids = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    for t in range(T):
        i_row = np.empty(k, np.int32)
        w_row = np.empty(k, np.float32)
        lib().haro_route_topk(np.ascontiguousarray(logits[t]), E, k, i_row, w_row)
        ids[t] = i_row
        w[t] = w_row
    lib().haro_set_exp_mode(0)
    return ids, w


Q6K_BLOCK_BYTES = 210


def q6k_dot(block: np.ndarray, x: np.ndarray) -> float:
    """har/crates/har-demo/src/bin/har-native-qwen3.rs:174-205"""
    return lib().haro_q6k_dot(np.ascontiguousarray(block, np.uint8),
                              np.ascontiguousarray(x, np.float32))


def q6k_matvec(w: np.ndarray, rows: int, K: int, x: np.ndarray) -> np.ndarray:
    """Q6_K rows [rows][K/256*210] times x: dot_quant_row's Q6_K arm per row
    (har-native-qwen3.rs:207-232), for every row of x [M][K] -> [M][rows]."""
    w = np.ascontiguousarray(w, np.uint8).reshape(-1)
    x = np.ascontiguousarray(x, np.float32).reshape(-1, K)
    out = np.empty((x.shape[0], rows), np.float32)
    for m in range(x.shape[0]):
        row = np.empty(rows, np.float32)
        lib().haro_q6k_matvec(w, rows, K, np.ascontiguousarray(x[m]), row)
        out[m] = row
    return out


def random_q6k(seed: int, rows: int, K: int, d_lo: float = 1e-3, d_hi: float = 4e-3) -> np.ndarray:
    """Seeded Q6_K test tensor [rows][K/256*210]: uniform random codes and
    int8 scales, d a random finite f16 in [d_lo, d_hi).  Any bytes are a
    valid Q6_K block apart from d, so no quantiser is involved."""
    rng = np.random.default_rng(seed)
    nb = rows * (K // QK_K)
    b = rng.integers(0, 256, size=(nb, Q6K_BLOCK_BYTES), dtype=np.uint8)
    d = rng.uniform(d_lo, d_hi, size=nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    b[:, 208:210] = d
    return b.reshape(rows, (K // QK_K) * Q6K_BLOCK_BYTES)


# ---- Q3_K (parity unpinned: the reference holds only the geometry,
# har/crates/har-model/src/lib.rs:591; the GGUF layout as ggml defines it) ----
Q3K_BLOCK_BYTES = 110


def q3k_scale(scales12: np.ndarray, s: int) -> int:
    return int(lib().haro_q3k_scale(np.ascontiguousarray(scales12, np.uint8), s))


def q3k_dequant_block(block: np.ndarray) -> np.ndarray:
    out = np.empty(256, np.float32)
    lib().haro_q3k_dequant_block(np.ascontiguousarray(block, np.uint8), out)
    return out


def q3k_matvec(w: np.ndarray, rows: int, K: int, x: np.ndarray) -> np.ndarray:
    """Q3_K rows [rows][K/256*110] times every row of x [M][K] -> [M][rows]."""
    w = np.ascontiguousarray(w, np.uint8).reshape(-1)
    x = np.ascontiguousarray(x, np.float32).reshape(-1, K)
    out = np.empty((x.shape[0], rows), np.float32)
    for m in range(x.shape[0]):
        row = np.empty(rows, np.float32)
        lib().haro_q3k_matvec(w, rows, K, np.ascontiguousarray(x[m]), row)
        out[m] = row
    return out


def random_q3k(seed: int, rows: int, K: int, d_lo: float = 1e-3, d_hi: float = 4e-3) -> np.ndarray:
    """Seeded Q3_K test tensor [rows][K/256*110]: uniform random bits and
    scales, d a random finite f16 in [d_lo, d_hi) (any other bytes decode)."""
    rng = np.random.default_rng(seed)
    nb = rows * (K // QK_K)
    b = rng.integers(0, 256, size=(nb, Q3K_BLOCK_BYTES), dtype=np.uint8)
    d = rng.uniform(d_lo, d_hi, size=nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    b[:, 108:110] = d
    return b.reshape(rows, (K // QK_K) * Q3K_BLOCK_BYTES)


def router_logits(gate_inp: np.ndarray, x: np.ndarray) -> np.ndarray:
    """routed_moe's self.matvec(ffn_gate_inp) on an F32 router
    (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:1168-1172, :154-163),
    per token row of x [T][H]; gate_inp [E][H]."""
    gate_inp = np.ascontiguousarray(gate_inp, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    E, H = gate_inp.shape
    out = np.empty((x.shape[0], E), np.float32)
    for t in range(x.shape[0]):
        row = np.empty(E, np.float32)
        lib().haro_router_logits(gate_inp, E, H, np.ascontiguousarray(x[t]), row)
        out[t] = row
    return out


def group_by_expert(ids: np.ndarray, E: int):
    """har/crates/har-serve/src/moe.rs:195-202"""
    ids = np.ascontiguousarray(ids, np.int32)
    T, k = ids.shape
    counts = np.empty(E, np.int32)
    offsets = np.empty(E + 1, np.int32)
    order = np.empty(T * k, np.int32)
    lib().haro_group_by_expert(T, k, E, ids.reshape(-1), counts, offsets, order)
    return counts, offsets, order


def q8k_quantize(x: np.ndarray) -> np.ndarray:
    """This project's Q8_K quantiser: rows of K f32 -> rows of K/256 x 292 B."""
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.reshape(-1, x.shape[-1]).shape
    out = np.empty((M, K // QK_K * Q8K_BLOCK_BYTES), np.uint8)
    for m in range(M):
        row = np.empty(K // QK_K * Q8K_BLOCK_BYTES, np.uint8)
        lib().haro_q8k_quantize(np.ascontiguousarray(x.reshape(M, K)[m]), K, row)
        out[m] = row
    return out


def q4k_gemv_q8k(w: np.ndarray, rows: int, K: int, xq: np.ndarray) -> np.ndarray:
    out = np.empty(rows, np.float32)
    lib().haro_q4k_gemv_q8k(np.ascontiguousarray(w, np.uint8).reshape(-1), rows, K,
                            np.ascontiguousarray(xq, np.uint8).reshape(-1), out)
    return out


def q4k_quantize(x: np.ndarray) -> np.ndarray:
    """This project's Q4_K quantiser (test-input generator)."""
    x = np.ascontiguousarray(x, np.float32)
    K = x.shape[-1]
    flat = x.reshape(-1, K)
    out = np.empty((flat.shape[0], K // QK_K * Q4K_BLOCK_BYTES), np.uint8)
    for r in range(flat.shape[0]):
        row = np.empty(K // QK_K * Q4K_BLOCK_BYTES, np.uint8)
        lib().haro_q4k_quantize_row(np.ascontiguousarray(flat[r]), K, row)
        out[r] = row
    return out.reshape(x.shape[:-1] + (K // QK_K * Q4K_BLOCK_BYTES,))


def lcg_values(count: int, seed: int) -> np.ndarray:
    """har/crates/har-serve/src/q4k.rs:109-120"""
    out = np.empty(count, np.float32)
    lib().haro_lcg_values(count, seed, out)
    return out


def normal_f32(seed: int, start: int, count: int, mean: float = 0.0, std: float = 1.0):
    out = np.empty(count, np.float32)
    lib().haro_normal_f32(seed, start, count, mean, std, out)
    return out


def gen_q4k(seed: int, rows: int, K: int, row0: int = 0, mean: float = 0.0,
            std: float = 0.02) -> np.ndarray:
    """rows x (K/256*144) bytes of N(mean, std) weights quantised to Q4_K."""
    out = np.empty(rows * (K // QK_K) * Q4K_BLOCK_BYTES, np.uint8)
    lib().haro_gen_q4k_rows(seed, row0, rows, K, mean, std, out)
    return out.reshape(rows, (K // QK_K) * Q4K_BLOCK_BYTES)


def zipf_routing(seed: int, T: int, E: int, k: int, s: float = 1.1):
    ids = np.empty(T * k, np.int32)
    w = np.empty(T * k, np.float32)
    lib().haro_zipf_routing(seed, T, E, k, s, ids, w)
    return ids.reshape(T, k), w.reshape(T, k)


def moe_ffn(w_gate, w_up, w_down, shared, sh_gate_inp, E, H, I, x, ids, weights,
            add_residual=False, threads=0, act="f32"):
    """compose_moe_route (har-native-qwen35moe.rs:979-1048) per token.

    shared = (gate, up, down) byte arrays or None; act "f32" is HAR's path,
    "q8k" the Q8_K-activation restatement."""
    x = np.ascontiguousarray(x, np.float32)
    ids = np.ascontiguousarray(ids, np.int32)
    weights = np.ascontiguousarray(weights, np.float32)
    T, k = ids.shape
    y = np.empty((T, H), np.float32)
    sg, su, sd = (None, None, None) if shared is None else tuple(
        np.ascontiguousarray(s, np.uint8) for s in shared)
    gi = None if sh_gate_inp is None else np.ascontiguousarray(sh_gate_inp, np.float32)
    fn = lib().haro_moe_ffn if act == "f32" else lib().haro_moe_ffn_q8k
    wg = np.ascontiguousarray(w_gate, np.uint8)
    wu = np.ascontiguousarray(w_up, np.uint8)
    wd = np.ascontiguousarray(w_down, np.uint8)
    fn(_ptr(wg), _ptr(wu), _ptr(wd), _ptr(sg), _ptr(su), _ptr(sd), _ptr(gi),
       E, H, I, T, k, _ptr(x), _ptr(ids), _ptr(weights), int(bool(add_residual)),
       _ptr(y), threads)
    return y


def online_cpus() -> int:
    return lib().haro_online_cpus()


def expf_restated(x: float) -> float:
    """glibc's expf restated (Nagy's table-driven method), as the GPU router computes it."""
    return lib().haro_expf_restated(x)


def exp2_table():
    """The restatement's 32-entry table of 2^(i/32) as IEEE double bit patterns."""
    out = (C.c_uint64 * 32)()
    lib().haro_exp2_table(out)
    return list(out)


def expf_mismatches(lo_bits: int, hi_bits: int):
    """(count, first bit pattern) of floats in [lo_bits, hi_bits] where the
    restatement differs from the host's expf (ctypes releases the GIL: callers
    may run ranges on several threads)."""
    first = C.c_uint32(0)
    n = lib().haro_expf_mismatches(lo_bits, hi_bits, C.byref(first))
    return int(n), int(first.value)
