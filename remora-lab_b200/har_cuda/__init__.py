"""har_cuda — Python host layer over libhar_cuda.so (the C ABI in include/har_cuda.h).

The CUDA library is the product; this module binds it with ctypes and mirrors
the reference's operator interface for the Q4_K MoE-FFN path (paths relative
to the leoinfer/remora-lab repository):

* ``CudaQ4KModel.matvec``      <- ``Q4KModel::matvec``            har/crates/har-serve/src/q4k.rs:170-188
* ``CudaQ4KModel.batch_step``  <- ``BatchStepModel::batch_step``   har/crates/har-serve/src/adapter.rs:28-72
* ``CudaMoeModel.expert_matvec``     <- ``expert_matvec``         har/crates/har-demo/src/bin/har-native-qwen35moe.rs:626-689
* ``CudaMoeModel.compose_moe_route`` <- ``compose_moe_route``     har-native-qwen35moe.rs:979-1048
* ``CudaMoeModel.routed_moe``        <- ``routed_moe``            har-native-qwen35moe.rs:1167-1215

Errors are fail-closed: every non-zero status raises ``HarCudaError`` (the
reference's GPU adapters panic, har/crates/har-serve/src/vulkan.rs:18-19).
There is no CPU fallback: importing this module without the built library, or
creating a context without a B200, raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libhar_cuda.so")

QK_K = 256
Q4K_BLOCK_BYTES = 144
Q8K_BLOCK_BYTES = 292
Q6K_BLOCK_BYTES = 210
Q3K_BLOCK_BYTES = 110
# GGML tensor type ids (har/crates/har-demo/src/bin/har-native-qwen35moe.rs:37-41)
GGML_F32, GGML_Q3_K, GGML_Q4_K, GGML_Q6_K = 0, 11, 12, 14
BLOCK_BYTES = {GGML_Q4_K: Q4K_BLOCK_BYTES, GGML_Q6_K: Q6K_BLOCK_BYTES, GGML_Q3_K: Q3K_BLOCK_BYTES}

OK = 0
CUDA_STREAM_LEGACY = 0x1  # cudaStreamLegacy: the legacy default stream's handle value
ERR_ARG, ERR_GEOMETRY, ERR_CUDA, ERR_NCCL, ERR_TIMEOUT = -1, -2, -3, -4, -5
ERR_NOT_INIT, ERR_OOM, ERR_UNSUPPORTED, ERR_DEVICE = -6, -7, -8, -9
STATUS_NAMES = {0: "OK", -1: "ARG", -2: "GEOMETRY", -3: "CUDA", -4: "NCCL", -5: "TIMEOUT",
                -6: "NOT_INIT", -7: "OOM", -8: "UNSUPPORTED", -9: "DEVICE"}

ACT_F32 = 0
ACT_Q8K = 1
MOE_ADD_RESIDUAL = 0x1
MOE_ACT_Q8K = 0x2
MOE_FORCE_GEMV = 0x4
MOE_FORCE_TC = 0x8
MOE_EMPTY_SLOTS = 0x10
MOE_TC_F16W = 0x20
MOE_DECODE = 0x40

# Every symbol include/har_cuda.h declares (tests check the library exports them).
EXPORTS = [
    "har_cuda_routed_moe_stack",
    "har_cuda_gguf_open", "har_cuda_gguf_close", "har_cuda_gguf_last_error",
    "har_cuda_gguf_header", "har_cuda_gguf_tensor_info", "har_cuda_gguf_find",
    "har_cuda_gguf_meta_u64", "har_cuda_gguf_meta_string", "har_cuda_weights_from_gguf",
    "har_cuda_gguf_read_f32", "har_cuda_moe_layer_from_gguf",
    "har_cuda_weights_upload", "har_cuda_weights_wrap", "har_cuda_q6k_gemv", "har_cuda_q3k_gemv",
    "har_cuda_router_logits", "har_cuda_route", "har_cuda_routed_moe",
    "har_cuda_abi_version", "har_cuda_ctx_create", "har_cuda_ctx_destroy", "har_cuda_last_error",
    "har_cuda_ctx_set_stream", "har_cuda_synchronize", "har_cuda_launch_count",
    "har_cuda_weights_upload_q4k", "har_cuda_weights_wrap_q4k", "har_cuda_weights_free",
    "har_cuda_weights_device_ptr", "har_cuda_q8k_quantize", "har_cuda_q4k_gemv",
    "har_cuda_route_topk", "har_cuda_group_by_expert", "har_cuda_moe_layer_create",
    "har_cuda_moe_layer_free", "har_cuda_moe_ffn", "har_cuda_moe_ffn_host", "har_cuda_moe_stack",
    "har_cuda_gen_q4k", "har_cuda_moe_stack_host", "har_cuda_profile_begin",
    "har_cuda_profile_end", "har_cuda_moe_ffn_noalloc", "har_cuda_ctx_set_tc_min_tokens",
    "har_cuda_ep_unique_id", "har_cuda_ep_create", "har_cuda_ep_free", "har_cuda_ep_moe_ffn",
    "har_cuda_ep_moe_stack", "har_cuda_ep_plan", "har_cuda_ep_combine",
    "har_cuda_ep_create_timeout", "har_cuda_ep_abort", "har_cuda_ep_set_p2p",
    "har_cuda_ep_exchange_mode",
    "har_cuda_slot_table_create", "har_cuda_slot_table_free", "har_cuda_slot_table_storage",
    "har_cuda_slot_table_last_error", "har_cuda_slot_reserve", "har_cuda_slot_mark_upload_submitted",
    "har_cuda_slot_upload", "har_cuda_slot_mark_ready", "har_cuda_slot_acquire",
    "har_cuda_slot_release", "har_cuda_slot_evict", "har_cuda_slot_table_snapshot",
]


class HarCudaError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"har_cuda status {status} ({STATUS_NAMES.get(status, '?')}): {message}")
        self.status = status


_lib = None


# expert-slot residency (har_cuda.h: HAR_CUDA_PROJ_*, HAR_CUDA_SLOT_*)
PROJ_GATE, PROJ_UP, PROJ_DOWN = 0, 1, 2
SLOT_FREE, SLOT_UPLOADING, SLOT_READY, SLOT_IN_FLIGHT = 0, 1, 2, 3


class SlotKey(C.Structure):
    """ExpertSlotKey (har/crates/har-vulkan/src/lib.rs:1239-1244)."""
    _fields_ = [("layer", C.c_uint32), ("expert_id", C.c_uint32), ("projection", C.c_uint32),
                ("generation", C.c_uint64)]


class SlotSnapshot(C.Structure):
    """ExpertSlotSnapshot (lib.rs:1253-1260)."""
    _fields_ = [("slot_id", C.c_uint32), ("key", SlotKey), ("state", C.c_int32),
                ("upload_epoch", C.c_uint64), ("last_use_epoch", C.c_uint64), ("ready", C.c_int32)]

    def as_dict(self):
        k = self.key
        return {"slot_id": self.slot_id, "key": (k.layer, k.expert_id, k.projection, k.generation),
                "state": self.state, "upload_epoch": self.upload_epoch,
                "last_use_epoch": self.last_use_epoch, "ready": bool(self.ready)}


def load_library() -> C.CDLL:
    """Load libhar_cuda.so; raises if it has not been built (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libhar_cuda.so not built at {LIB_PATH}; run remora-lab_b200/build.py")
    # The library links libnccl.so.2.  Loaded first, it would pull in the
    # system NCCL, which lacks symbols torch's own (newer) NCCL provides and
    # makes a later `import torch` fail; with torch loaded first both share
    # torch's NCCL.
    try:
        import torch  # noqa: F401
    except ImportError:
        pass
    L = C.CDLL(LIB_PATH)
    vp, i32, i64, u32, u64 = C.c_void_p, C.c_int32, C.c_int64, C.c_uint32, C.c_uint64
    pp = C.POINTER(C.c_void_p)
    sigs = {
        "har_cuda_abi_version": (i32, []),
        "har_cuda_ctx_create": (i32, [i32, pp]),
        "har_cuda_ctx_destroy": (i32, [vp]),
        "har_cuda_last_error": (i32, [vp, C.c_char_p, C.c_size_t]),
        "har_cuda_ctx_set_stream": (i32, [vp, vp]),
        "har_cuda_ctx_set_tc_min_tokens": (i32, [vp, i32]),
        "har_cuda_ep_unique_id": (i32, [vp, C.c_size_t]),
        "har_cuda_ep_create": (i32, [vp, vp, C.c_size_t, i32, i32, pp]),
        "har_cuda_ep_free": (i32, [vp]),
        "har_cuda_ep_create_timeout": (i32, [vp, vp, C.c_size_t, i32, i32, i64, pp]),
        "har_cuda_ep_abort": (i32, [vp]),
        "har_cuda_ep_set_p2p": (i32, [vp, i32]),
        "har_cuda_ep_exchange_mode": (i32, [vp]),
        "har_cuda_ep_moe_ffn": (i32, [vp, vp, vp, vp, vp, vp, i64, i32, vp, vp, vp, u32]),
        "har_cuda_ep_moe_stack": (i32, [vp, vp, vp, vp, vp, i32, vp, i64, i32, vp, vp, vp, u32]),
        "har_cuda_ep_plan": (i32, [vp, vp, i64, i64, i32, vp, vp, i32, i32, vp, vp, vp]),
        "har_cuda_ep_combine": (i32, [vp, vp, i64, i64, i32, vp, vp, u32, vp]),
        "har_cuda_synchronize": (i32, [vp, i64]),
        "har_cuda_launch_count": (i64, [vp]),
        "har_cuda_weights_upload_q4k": (i32, [vp, vp, i64, i64, i64, pp]),
        "har_cuda_weights_wrap_q4k": (i32, [vp, vp, i64, i64, i64, pp]),
        "har_cuda_weights_free": (i32, [vp]),
        "har_cuda_weights_upload": (i32, [vp, i32, vp, i64, i64, i64, pp]),
        "har_cuda_weights_wrap": (i32, [vp, i32, vp, i64, i64, i64, pp]),
        "har_cuda_q6k_gemv": (i32, [vp, vp, i64, vp, i64, vp]),
        "har_cuda_q3k_gemv": (i32, [vp, vp, i64, vp, i64, vp]),
        "har_cuda_gguf_open": (i32, [C.c_char_p, C.c_char_p, C.c_size_t, pp]),
        "har_cuda_gguf_close": (i32, [vp]),
        "har_cuda_gguf_last_error": (i32, [vp, C.c_char_p, C.c_size_t]),
        "har_cuda_gguf_header": (i32, [vp, C.POINTER(C.c_uint32), C.POINTER(u64),
                                       C.POINTER(u64), C.POINTER(u64), C.POINTER(u64)]),
        "har_cuda_gguf_tensor_info": (i32, [vp, i64, C.c_char_p, C.c_size_t,
                                            C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                            C.POINTER(u64), C.POINTER(u64), C.POINTER(u64)]),
        "har_cuda_gguf_find": (i64, [vp, C.c_char_p]),
        "har_cuda_gguf_meta_u64": (i32, [vp, C.c_char_p, C.POINTER(u64)]),
        "har_cuda_gguf_meta_string": (i32, [vp, C.c_char_p, C.c_char_p, C.c_size_t]),
        "har_cuda_weights_from_gguf": (i32, [vp, vp, C.c_char_p, pp]),
        "har_cuda_gguf_read_f32": (i32, [vp, vp, C.c_char_p, vp, i64]),
        "har_cuda_moe_layer_from_gguf": (i32, [vp, vp, i32, pp]),
        "har_cuda_weights_device_ptr": (vp, [vp]),
        "har_cuda_q8k_quantize": (i32, [vp, vp, i64, i64, vp]),
        "har_cuda_q4k_gemv": (i32, [vp, vp, i64, vp, i32, i64, vp]),
        "har_cuda_route_topk": (i32, [vp, vp, i64, i32, i32, vp, vp]),
        "har_cuda_router_logits": (i32, [vp, vp, i32, i64, vp, i64, vp]),
        "har_cuda_route": (i32, [vp, vp, i32, i64, vp, i64, i32, vp, vp]),
        "har_cuda_routed_moe": (i32, [vp, vp, vp, vp, i64, i32, vp, vp, vp, u32]),
        "har_cuda_routed_moe_stack": (i32, [vp, vp, i32, vp, vp, i64, i32, vp, vp, vp, u32]),
        "har_cuda_group_by_expert": (i32, [vp, vp, i64, i32, i32, vp, vp, vp]),
        "har_cuda_moe_layer_create": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, pp]),
        "har_cuda_moe_layer_free": (i32, [vp]),
        "har_cuda_moe_ffn": (i32, [vp, vp, vp, i64, i32, vp, vp, vp, u32]),
        "har_cuda_moe_ffn_host": (i32, [vp, vp, vp, i64, i32, vp, vp, vp, u32]),
        "har_cuda_moe_stack": (i32, [vp, vp, i32, vp, i64, i32, vp, vp, vp, u32]),
        "har_cuda_gen_q4k": (i32, [vp, vp, i64, i64, u64, i64, C.c_float, C.c_float]),
        "har_cuda_moe_stack_host": (i32, [vp, vp, i32, vp, i64, i32, vp, vp, vp, u32]),
        "har_cuda_profile_begin": (i32, [vp]),
        "har_cuda_moe_ffn_noalloc": (i32, [vp, vp, vp, i64, i32, vp, vp, vp, u32]),
        "har_cuda_profile_end": (i32, [vp, C.c_char_p, C.c_size_t, vp, i64, C.POINTER(C.c_int64)]),
        "har_cuda_slot_table_create": (i32, [vp, u32, u64, pp]),
        "har_cuda_slot_table_free": (i32, [vp]),
        "har_cuda_slot_table_storage": (i32, [vp, pp, C.POINTER(u64)]),
        "har_cuda_slot_table_last_error": (i32, [vp, C.c_char_p, C.c_size_t]),
        "har_cuda_slot_reserve": (i32, [vp, C.POINTER(SlotKey), C.POINTER(u32)]),
        "har_cuda_slot_mark_upload_submitted": (i32, [vp, u32, vp]),
        "har_cuda_slot_upload": (i32, [vp, u32, vp, u64]),
        "har_cuda_slot_mark_ready": (i32, [vp, u32, vp]),
        "har_cuda_slot_acquire": (i32, [vp, C.POINTER(SlotKey), C.POINTER(SlotSnapshot)]),
        "har_cuda_slot_release": (i32, [vp, u32, vp]),
        "har_cuda_slot_evict": (i32, [vp, u32, vp]),
        "har_cuda_slot_table_snapshot": (i32, [vp, C.POINTER(SlotSnapshot), u32, C.POINTER(u32)]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _dptr(t) -> int:
    """Device pointer of a torch CUDA tensor (None -> NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise HarCudaError(ERR_ARG, "expected a CUDA tensor")
    if not t.is_contiguous():
        raise HarCudaError(ERR_ARG, "expected a contiguous tensor")
    return t.data_ptr()


def _hptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


class Context:
    """One device + one stream (har/crates/har-vulkan/src/lib.rs:236 Device::open).

    By default kernels run on torch's current stream of the device, so they
    order with the caller's torch work."""

    def __init__(self, device: int = 0, use_torch_stream: bool = True):
        self.lib = load_library()
        h = C.c_void_p()
        st = self.lib.har_cuda_ctx_create(device, C.byref(h))
        if st != OK:
            raise HarCudaError(st, f"ctx_create(device={device}) failed")
        self.handle = h
        self.device = device
        if use_torch_stream:
            self.bind_torch_stream()

    def bind_torch_stream(self):
        """Launch on torch's current stream of the device.  torch's default
        stream is the legacy default stream, whose handle is 0; the ABI reads
        NULL as "the context's own stream", so it is passed as
        cudaStreamLegacy (0x1), which orders with torch's default-stream work."""
        import torch
        s = torch.cuda.current_stream(self.device)
        self.check(self.lib.har_cuda_ctx_set_stream(self.handle,
                                                    C.c_void_p(s.cuda_stream or CUDA_STREAM_LEGACY)))

    def set_tc_min_tokens(self, n: int):
        """Experts with >= n tokens take the tensor-core kernels (0 = default)."""
        self.check(self.lib.har_cuda_ctx_set_tc_min_tokens(self.handle, n))

    def last_error(self) -> str:
        buf = C.create_string_buffer(1024)
        self.lib.har_cuda_last_error(self.handle, buf, 1024)
        return buf.value.decode(errors="replace")

    def check(self, status: int):
        if status != OK:
            raise HarCudaError(status, self.last_error())

    def synchronize(self, timeout_ms: int = 60000):
        self.check(self.lib.har_cuda_synchronize(self.handle, timeout_ms))

    @property
    def launch_count(self) -> int:
        return int(self.lib.har_cuda_launch_count(self.handle))

    def close(self):
        if getattr(self, "handle", None):
            self.lib.har_cuda_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- weights --------------------------------------------------------
    def upload_q4k(self, host_bytes: np.ndarray, E: int, N: int, K: int) -> "Q4KWeights":
        host_bytes = np.ascontiguousarray(host_bytes, np.uint8)
        if host_bytes.size != E * N * (K // QK_K) * Q4K_BLOCK_BYTES:
            raise HarCudaError(ERR_GEOMETRY, "Q4_K byte count does not match E*N*K/256*144")
        h = C.c_void_p()
        self.check(self.lib.har_cuda_weights_upload_q4k(self.handle, _hptr(host_bytes), E, N, K,
                                                        C.byref(h)))
        return Q4KWeights(self, h, E, N, K)

    def upload(self, ggml_type: int, host_bytes: np.ndarray, E: int, N: int,
               K: int) -> "Q4KWeights":
        """Upload a GGUF block tensor [E][N][K/256] of a supported type."""
        host_bytes = np.ascontiguousarray(host_bytes, np.uint8)
        if ggml_type not in BLOCK_BYTES:
            raise HarCudaError(ERR_UNSUPPORTED, f"GGML type {ggml_type}")
        if host_bytes.size != E * N * (K // QK_K) * BLOCK_BYTES[ggml_type]:
            raise HarCudaError(ERR_GEOMETRY, "byte count does not match E*N*K/256*block_bytes")
        h = C.c_void_p()
        self.check(self.lib.har_cuda_weights_upload(self.handle, ggml_type, _hptr(host_bytes), E,
                                                    N, K, C.byref(h)))
        return Q4KWeights(self, h, E, N, K, ggml_type)

    def wrap(self, ggml_type: int, dev_tensor, E: int, N: int, K: int) -> "Q4KWeights":
        h = C.c_void_p()
        self.check(self.lib.har_cuda_weights_wrap(self.handle, ggml_type, _dptr(dev_tensor), E, N,
                                                  K, C.byref(h)))
        w = Q4KWeights(self, h, E, N, K, ggml_type)
        w.keepalive = dev_tensor
        return w

    def wrap_q4k(self, dev_tensor, E: int, N: int, K: int) -> "Q4KWeights":
        h = C.c_void_p()
        self.check(self.lib.har_cuda_weights_wrap_q4k(self.handle, _dptr(dev_tensor), E, N, K,
                                                      C.byref(h)))
        w = Q4KWeights(self, h, E, N, K)
        w.keepalive = dev_tensor
        return w

    def gen_q4k(self, dev_tensor, rows: int, K: int, seed: int, row0: int = 0,
                mean: float = 0.0, std: float = 0.02):
        self.check(self.lib.har_cuda_gen_q4k(self.handle, _dptr(dev_tensor), rows, K, seed, row0,
                                             mean, std))

    # ---- kernels ----------------------------------------------------------
    def q8k_quantize(self, x, out):
        M, K = x.shape
        self.check(self.lib.har_cuda_q8k_quantize(self.handle, _dptr(x), M, K, _dptr(out)))
        return out

    def q4k_gemv(self, w: "Q4KWeights", expert: int, x, act_kind: int, M: int, y):
        self.check(self.lib.har_cuda_q4k_gemv(self.handle, w.handle, expert, _dptr(x), act_kind, M,
                                              _dptr(y)))
        return y

    # ---- GGUF ---------------------------------------------------------------
    def weights_from_gguf(self, g: "Gguf", name: str) -> "Q4KWeights":
        """Upload a Q3_K/Q4_K/Q6_K tensor of a GGUF file into the device layout."""
        h = C.c_void_p()
        self.check(self.lib.har_cuda_weights_from_gguf(self.handle, g.handle, name.encode(),
                                                       C.byref(h)))
        info = g.tensor(name)
        d = info["dims"]
        E = d[2] if len(d) == 3 else 1
        return Q4KWeights(self, h, E, d[1], d[0], info["type"])

    def gguf_read_f32(self, g: "Gguf", name: str, dst):
        self.check(self.lib.har_cuda_gguf_read_f32(self.handle, g.handle, name.encode(), _dptr(dst),
                                                   dst.numel()))
        return dst

    def moe_layer_from_gguf(self, g: "Gguf", layer: int) -> "MoeLayer":
        """blk.<layer>'s expert, shared-expert and router tensors as one layer
        that owns them (har-native-qwen35moe.rs:979-1048,1167-1215)."""
        h = C.c_void_p()
        self.check(self.lib.har_cuda_moe_layer_from_gguf(self.handle, g.handle, layer, C.byref(h)))
        H, I, E = g.tensor(f"blk.{layer}.ffn_gate_exps.weight")["dims"]
        ml = MoeLayer(self, h, None, E, H, I)
        ml.shared = g.find(f"blk.{layer}.ffn_gate_shexp.weight") >= 0
        return ml

    def q3k_gemv(self, w: "Q4KWeights", expert: int, x, M: int, y):
        """y [M][N] = W_e x for Q3_K weights and f32 activations x [M][K]."""
        self.check(self.lib.har_cuda_q3k_gemv(self.handle, w.handle, expert, _dptr(x), M,
                                              _dptr(y)))
        return y

    def q6k_gemv(self, w: "Q4KWeights", expert: int, x, M: int, y):
        """y [M][N] = W_e x for Q6_K weights and f32 activations x [M][K]."""
        self.check(self.lib.har_cuda_q6k_gemv(self.handle, w.handle, expert, _dptr(x), M,
                                              _dptr(y)))
        return y

    def route_topk(self, logits, k: int, ids, weights):
        T, E = logits.shape
        self.check(self.lib.har_cuda_route_topk(self.handle, _dptr(logits), T, E, k, _dptr(ids),
                                                _dptr(weights)))
        return ids, weights

    def router_logits(self, gate_inp, x, logits):
        """routed_moe's router GEMV, self.matvec(ffn_gate_inp)
        (har-native-qwen35moe.rs:1168-1172): gate_inp f32 [E][H], x f32
        [T][H] -> logits f32 [T][E], bit-exact with the reference."""
        E, H = gate_inp.shape
        T = x.shape[0]
        if x.shape[1] != H or tuple(logits.shape) != (T, E):
            raise HarCudaError(ERR_GEOMETRY, "router_logits: x [T][H], logits [T][E]")
        self.check(self.lib.har_cuda_router_logits(self.handle, _dptr(gate_inp), E, H, _dptr(x),
                                                   T, _dptr(logits)))
        return logits

    def route(self, gate_inp, x, k: int, ids, weights):
        """routed_moe's selection (har-native-qwen35moe.rs:1167-1204) from the
        token rows: router GEMV, softmax over all E, top-k, renormalise."""
        E, H = gate_inp.shape
        T = x.shape[0]
        if x.shape[1] != H or tuple(ids.shape) != (T, k) or tuple(weights.shape) != (T, k):
            raise HarCudaError(ERR_GEOMETRY, "route: x [T][H], ids/weights [T][k]")
        self.check(self.lib.har_cuda_route(self.handle, _dptr(gate_inp), E, H, _dptr(x), T, k,
                                           _dptr(ids), _dptr(weights)))
        return ids, weights

    def routed_moe(self, layer: "MoeLayer", gate_inp, x, k: int, ids, weights, y,
                   flags: int = 0):
        """routed_moe (har-native-qwen35moe.rs:1167-1215): route x with the
        f32 router gate_inp [E][H], write the route record to ids/weights
        [T][k] and the layer's output to y [T][H]."""
        T = x.shape[0]
        if tuple(ids.shape) != (T, k) or tuple(weights.shape) != (T, k):
            raise HarCudaError(ERR_GEOMETRY, "routed_moe: ids/weights [T][k]")
        self.check(self.lib.har_cuda_routed_moe(self.handle, layer.handle, _dptr(gate_inp),
                                                _dptr(x), T, k, _dptr(ids), _dptr(weights),
                                                _dptr(y), flags))
        return y

    def routed_moe_stack(self, layers, routers, x, k: int, ids, weights, y, flags: int = 0):
        """L routed layers in one call (har_cuda_routed_moe_stack): routers is a
        list of f32 [E][H] device tensors or None entries (the layer's own
        router), or None for all; ids/weights [L][T][k] receive the route
        records."""
        L = len(layers)
        T = x.shape[0]
        if tuple(ids.shape) != (L, T, k) or tuple(weights.shape) != (L, T, k):
            raise HarCudaError(ERR_GEOMETRY, "routed_moe_stack: ids/weights [L][T][k]")
        arr = (C.c_void_p * L)(*[l.handle for l in layers])
        rt = None
        if routers is not None:
            if len(routers) != L:
                raise HarCudaError(ERR_GEOMETRY, "routed_moe_stack: one router entry per layer")
            rt = (C.c_void_p * L)(*[_dptr(r) for r in routers])
        self.check(self.lib.har_cuda_routed_moe_stack(self.handle, arr, L, rt, _dptr(x), T, k,
                                                      _dptr(ids), _dptr(weights), _dptr(y), flags))
        return y

    def group_by_expert(self, ids, E: int, counts, offsets, order):
        T, k = ids.shape
        self.check(self.lib.har_cuda_group_by_expert(self.handle, _dptr(ids), T, k, E,
                                                     _dptr(counts), _dptr(offsets), _dptr(order)))

    def moe_layer(self, gate, up, down, shared=None, sh_gate_inp=None) -> "MoeLayer":
        sg, su, sd = (None, None, None) if shared is None else shared
        h = C.c_void_p()
        self.check(self.lib.har_cuda_moe_layer_create(
            self.handle, gate.handle, up.handle, down.handle,
            sg.handle if sg else None, su.handle if su else None, sd.handle if sd else None,
            _dptr(sh_gate_inp), C.byref(h)))
        return MoeLayer(self, h, (gate, up, down, sg, su, sd, sh_gate_inp), gate.E, gate.K, gate.N)

    def moe_ffn(self, layer: "MoeLayer", x, ids, weights, y, flags: int = 0):
        T, k = ids.shape
        self.check(self.lib.har_cuda_moe_ffn(self.handle, layer.handle, _dptr(x), T, k, _dptr(ids),
                                             _dptr(weights), _dptr(y), flags))
        return y

    def moe_ffn_noalloc(self, layer: "MoeLayer", x, ids, weights, y, flags: int = 0):
        """moe_ffn on the library's static device scratch: allocates nothing
        (for callers that cannot call cudaMalloc; see include/har_cuda.h)."""
        T, k = ids.shape
        self.check(self.lib.har_cuda_moe_ffn_noalloc(self.handle, layer.handle, _dptr(x), T, k,
                                                     _dptr(ids), _dptr(weights), _dptr(y), flags))
        return y

    def moe_ffn_host(self, layer: "MoeLayer", x: np.ndarray, ids: np.ndarray,
                     weights: np.ndarray, flags: int = 0) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        ids = np.ascontiguousarray(ids, np.int32)
        weights = np.ascontiguousarray(weights, np.float32)
        T, k = ids.shape
        y = np.empty_like(x)
        self.check(self.lib.har_cuda_moe_ffn_host(self.handle, layer.handle, _hptr(x), T, k,
                                                  _hptr(ids), _hptr(weights), _hptr(y), flags))
        return y

    def moe_stack_host(self, layers, x: np.ndarray, ids: np.ndarray, weights: np.ndarray,
                       flags: int = 0) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        ids = np.ascontiguousarray(ids, np.int32)
        weights = np.ascontiguousarray(weights, np.float32)
        L, T, k = ids.shape
        arr = (C.c_void_p * L)(*[l.handle.value for l in layers])
        y = np.empty_like(x)
        self.check(self.lib.har_cuda_moe_stack_host(self.handle, arr, L, _hptr(x), T, k,
                                                    _hptr(ids), _hptr(weights), _hptr(y), flags))
        return y

    def profile_begin(self):
        self.check(self.lib.har_cuda_profile_begin(self.handle))

    def profile_end(self, cap: int = 1 << 16):
        """[(kernel name, milliseconds)] for every launch since profile_begin."""
        names = C.create_string_buffer(cap * 32)
        ms = np.zeros(cap, np.float32)
        n = C.c_int64()
        self.check(self.lib.har_cuda_profile_end(self.handle, names, len(names), _hptr(ms), cap,
                                                 C.byref(n)))
        lst = names.value.decode().split("\n")[:n.value]
        return list(zip(lst, ms[:n.value].tolist()))

    def moe_stack(self, layers, x, ids, weights, y, flags: int = 0):
        L = len(layers)
        arr = (C.c_void_p * L)(*[l.handle.value for l in layers])
        _, T, k = ids.shape
        self.check(self.lib.har_cuda_moe_stack(self.handle, arr, L, _dptr(x), T, k, _dptr(ids),
                                               _dptr(weights), _dptr(y), flags))
        return y

    # ---- expert parallelism -------------------------------------------------
    def ep_create(self, unique_id: bytes, world: int, rank: int,
                  timeout_ms: int = 300000) -> "EpComm":
        """Collective over `world` ranks: join the NCCL communicator on this
        device; raises HarCudaError (ERR_TIMEOUT) when not every rank joins
        within timeout_ms (the same bound then holds for each exchange)."""
        buf = (C.c_uint8 * len(unique_id)).from_buffer_copy(unique_id)
        h = C.c_void_p()
        self.check(self.lib.har_cuda_ep_create_timeout(self.handle, buf, len(unique_id), world,
                                                       rank, timeout_ms, C.byref(h)))
        return EpComm(self, h, world, rank)

    def ep_moe_ffn(self, ep: "EpComm", local: "MoeLayer", shared, gate_inp, x, ids, weights, y,
                   flags: int = 0):
        T, k = ids.shape
        self.check(self.lib.har_cuda_ep_moe_ffn(
            self.handle, ep.handle, local.handle, shared.handle if shared else None,
            _dptr(gate_inp), _dptr(x), T, k, _dptr(ids), _dptr(weights), _dptr(y), flags))
        return y

    def ep_moe_stack(self, ep: "EpComm", locals_, shareds, gate_inps, x, ids, weights, y,
                     flags: int = 0):
        L = len(locals_)
        la = (C.c_void_p * L)(*[l.handle.value for l in locals_])
        sa = (C.c_void_p * L)(*[s.handle.value for s in shareds]) if shareds else None
        ga = (C.c_void_p * L)(*[_dptr(g) for g in gate_inps]) if gate_inps else None
        _, T, k = ids.shape
        self.check(self.lib.har_cuda_ep_moe_stack(
            self.handle, ep.handle, la, sa, ga, L, _dptr(x), T, k, _dptr(ids), _dptr(weights),
            _dptr(y), flags))
        return y

    def ep_plan(self, x, ids, weights, E: int, world: int, sx, sids, sw):
        """ep_plan_kernel alone: the dispatch rows [world*T] for every destination."""
        T, k = ids.shape
        self.check(self.lib.har_cuda_ep_plan(self.handle, _dptr(x), x.shape[1], T, k, _dptr(ids),
                                             _dptr(weights), E, world, _dptr(sx), _dptr(sids),
                                             _dptr(sw)))

    def ep_combine(self, x, world: int, shared, back, y, flags: int = 0):
        """ep_combine_kernel alone: y = residual + shared + back[0] + ... + back[world-1]."""
        T, H = x.shape
        self.check(self.lib.har_cuda_ep_combine(self.handle, _dptr(x), H, T, world,
                                                _dptr(shared) if shared is not None else None,
                                                _dptr(back), flags, _dptr(y)))


def ep_unique_id() -> bytes:
    """An NCCL unique id for har_cuda_ep_create (made on one rank, sent to all)."""
    lib = load_library()
    buf = (C.c_uint8 * 128)()
    st = lib.har_cuda_ep_unique_id(buf, 128)
    if st != 0:
        raise HarCudaError(st, "ncclGetUniqueId failed")
    return bytes(buf)


def expert_range(E: int, world: int, rank: int):
    """Routed experts [lo, hi) held by `rank` of `world` (E divisible by world)."""
    if world < 1 or not 0 <= rank < world or E % world:
        raise ValueError(f"cannot shard {E} experts over {world} ranks (rank {rank})")
    el = E // world
    return rank * el, (rank + 1) * el


class EpComm:
    """An expert-parallel communicator (one per rank and context): NCCL, plus
    the peer-memory windows mapped on first use; free it explicitly, on every
    rank, after the last collective call (the free is collective too)."""

    def __init__(self, ctx: "Context", handle, world: int, rank: int):
        self.ctx, self.handle, self.world, self.rank = ctx, handle, world, rank

    def set_p2p(self, on: bool):
        """Peer-memory exchange (opt-in) or the NCCL rounds (default); same value on every rank."""
        st = self.ctx.lib.har_cuda_ep_set_p2p(self.handle, 1 if on else 0)
        if st != 0:
            raise HarCudaError(st, "ep_set_p2p failed")

    @property
    def exchange_mode(self) -> int:
        """1 peer memory, 0 NCCL (chosen or not yet set up), -1 NCCL (windows unmappable)."""
        return int(self.ctx.lib.har_cuda_ep_exchange_mode(self.handle))

    def abort(self):
        """Abort the communicator (its in-flight exchanges end with an error)."""
        if self.handle:
            self.ctx.lib.har_cuda_ep_abort(self.handle)

    def free(self):
        if self.handle:
            self.ctx.lib.har_cuda_ep_free(self.handle)
            self.handle = None


class Q4KWeights:
    """A device-resident block tensor [E][N][K/256] (GGUF `*_exps` layout),
    Q4_K unless ggml_type says otherwise."""

    def __init__(self, ctx: Context, handle, E, N, K, ggml_type: int = GGML_Q4_K):
        self.ctx, self.handle, self.E, self.N, self.K = ctx, handle, E, N, K
        self.ggml_type = ggml_type
        self.row_bytes = K // QK_K * BLOCK_BYTES[ggml_type]
        self.keepalive = None

    @property
    def nbytes(self) -> int:
        return self.E * self.N * self.row_bytes

    def free(self):
        if self.handle:
            self.ctx.lib.har_cuda_weights_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Gguf:
    """A GGUF file's directory (GgufReader::inspect, har/crates/har-model/src/lib.rs:126-399).
    Host-only: opening and querying need no GPU."""

    def __init__(self, path: str):
        self.lib = load_library()
        h = C.c_void_p()
        err = C.create_string_buffer(512)
        st = self.lib.har_cuda_gguf_open(os.fsencode(path), err, 512, C.byref(h))
        if st != OK:
            raise HarCudaError(st, err.value.decode(errors="replace"))
        self.handle = h
        v, tc, mc, al, do = (C.c_uint32(), C.c_uint64(), C.c_uint64(), C.c_uint64(), C.c_uint64())
        self.lib.har_cuda_gguf_header(h, C.byref(v), C.byref(tc), C.byref(mc), C.byref(al),
                                      C.byref(do))
        self.version, self.tensor_count, self.metadata_count = v.value, tc.value, mc.value
        self.alignment, self.data_offset = al.value, do.value

    def _err(self) -> str:
        buf = C.create_string_buffer(512)
        self.lib.har_cuda_gguf_last_error(self.handle, buf, 512)
        return buf.value.decode(errors="replace")

    def tensor_info(self, index: int) -> dict:
        name = C.create_string_buffer(4096)
        t, r = C.c_uint32(), C.c_uint32()
        dims = (C.c_uint64 * 16)()
        off, pay = C.c_uint64(), C.c_uint64()
        st = self.lib.har_cuda_gguf_tensor_info(self.handle, index, name, 4096, C.byref(t),
                                                C.byref(r), dims, C.byref(off), C.byref(pay))
        if st != OK:
            raise HarCudaError(st, self._err())
        return {"name": name.value.decode(), "type": t.value, "dims": list(dims[:r.value]),
                "file_offset": off.value, "payload_bytes": pay.value}

    def tensors(self):
        return [self.tensor_info(i) for i in range(self.tensor_count)]

    def find(self, name: str) -> int:
        return int(self.lib.har_cuda_gguf_find(self.handle, name.encode()))

    def tensor(self, name: str) -> dict:
        i = self.find(name)
        if i < 0:
            raise HarCudaError(ERR_ARG, f"no tensor {name}")
        return self.tensor_info(i)

    def meta_u64(self, key: str):
        v = C.c_uint64()
        st = self.lib.har_cuda_gguf_meta_u64(self.handle, key.encode(), C.byref(v))
        return v.value if st == OK else None

    def meta_string(self, key: str):
        buf = C.create_string_buffer(4096)
        st = self.lib.har_cuda_gguf_meta_string(self.handle, key.encode(), buf, 4096)
        return buf.value.decode(errors="replace") if st == OK else None

    def close(self):
        if getattr(self, "handle", None):
            self.lib.har_cuda_gguf_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class MoeLayer:
    def __init__(self, ctx: Context, handle, refs, E: int = 0, H: int = 0, I: int = 0):
        self.ctx, self.handle, self.refs = ctx, handle, refs
        self.E, self.H, self.I = E, H, I
        self.shared = refs is None or refs[3] is not None

    def expert_bytes(self) -> int:
        """Q4_K bytes of one expert's gate, up and down."""
        return 3 * self.I * (self.H // QK_K) * Q4K_BLOCK_BYTES

    def free(self):
        if self.handle:
            self.ctx.lib.har_cuda_moe_layer_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def _event_ptr(event):
    """A torch.cuda.Event (or a raw cudaEvent_t as int) as void*, None -> NULL."""
    if event is None:
        return None
    return C.c_void_p(event.cuda_event if hasattr(event, "cuda_event") else int(event))


class SlotTable:
    """ExpertSlotTable (har/crates/har-vulkan/src/lib.rs:1233-1460) through the
    C ABI: `slot_count` device slots of `slot_bytes` each (ctx None: the state
    machine alone, no storage, events None).  Errors raise HarCudaError with the
    reference's message."""

    def __init__(self, ctx: "Context", slot_count: int, slot_bytes: int):
        self.ctx = ctx
        self.lib = ctx.lib if ctx is not None else load_library()
        h = C.c_void_p()
        st = self.lib.har_cuda_slot_table_create(ctx.handle if ctx is not None else None, slot_count,
                                                 slot_bytes, C.byref(h))
        if st:
            raise HarCudaError(st, "slot table: create failed")
        self.handle, self.slot_count, self.slot_bytes = h, slot_count, slot_bytes

    def _check(self, st: int):
        if st:
            buf = C.create_string_buffer(512)
            self.lib.har_cuda_slot_table_last_error(self.handle, buf, len(buf))
            raise HarCudaError(st, buf.value.decode())

    @staticmethod
    def key(layer: int, expert: int, projection: int, generation: int = 1) -> SlotKey:
        return SlotKey(layer, expert, projection, generation)

    def storage(self):
        """(device address, bytes) of the slots' storage (0 without a context)."""
        p, n = C.c_void_p(), C.c_uint64()
        self._check(self.lib.har_cuda_slot_table_storage(self.handle, C.byref(p), C.byref(n)))
        return p.value or 0, n.value

    def reserve(self, key: SlotKey) -> int:
        sid = C.c_uint32()
        self._check(self.lib.har_cuda_slot_reserve(self.handle, C.byref(key), C.byref(sid)))
        return sid.value

    def mark_upload_submitted(self, slot_id: int, event=None):
        self._check(self.lib.har_cuda_slot_mark_upload_submitted(self.handle, slot_id, _event_ptr(event)))

    def upload(self, slot_id: int, data: np.ndarray):
        data = np.ascontiguousarray(data)
        self._check(self.lib.har_cuda_slot_upload(self.handle, slot_id, _hptr(data), data.nbytes))
        self._keep = data  # the copy is asynchronous: keep the source until the next upload

    def mark_ready(self, slot_id: int, event=None):
        self._check(self.lib.har_cuda_slot_mark_ready(self.handle, slot_id, _event_ptr(event)))

    def acquire(self, key: SlotKey) -> dict:
        out = SlotSnapshot()
        self._check(self.lib.har_cuda_slot_acquire(self.handle, C.byref(key), C.byref(out)))
        return out.as_dict()

    def release(self, slot_id: int, event=None):
        self._check(self.lib.har_cuda_slot_release(self.handle, slot_id, _event_ptr(event)))

    def evict(self, slot_id: int, event=None):
        self._check(self.lib.har_cuda_slot_evict(self.handle, slot_id, _event_ptr(event)))

    def snapshot(self) -> list:
        arr = (SlotSnapshot * self.slot_count)()
        n = C.c_uint32()
        self._check(self.lib.har_cuda_slot_table_snapshot(self.handle, arr, self.slot_count, C.byref(n)))
        return [arr[i].as_dict() for i in range(n.value)]

    def free(self):
        if self.handle:
            self.lib.har_cuda_slot_table_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class SlottedMoeLayer:
    """A MoE layer whose E experts live in host memory with at most n_slots of
    them on the device: the host side of expert-slot residency (the role of
    ExpertSlotTable in HAR's serving path).  One SlotTable per projection keeps
    an expert's gate, up and down at the same slot index; the tables' storage
    is wrapped as an n_slots-expert Q4_K layer, and a call maps its expert ids
    to slot ids, so the kernels are the ordinary ones.  Missing experts evict
    the least recently used slots the call does not need (epochs from the
    tables' snapshots); slots are acquired for the dispatch and released once
    its event has completed (at the next call)."""

    def __init__(self, ctx: "Context", host_gate, host_up, host_down, E: int, H: int, I: int,
                 n_slots: int, layer_id: int = 0, shared=None, sh_gate_inp=None):
        self.ctx, self.E, self.H, self.I, self.n_slots, self.layer_id = ctx, E, H, I, n_slots, layer_id
        pb = I * (H // QK_K) * Q4K_BLOCK_BYTES
        assert H * (I // QK_K) * Q4K_BLOCK_BYTES == pb
        self.host = [np.ascontiguousarray(h).reshape(E, pb) for h in (host_gate, host_up, host_down)]
        self.tables = [SlotTable(ctx, n_slots, pb) for _ in range(3)]
        views = []
        for p, (N, K) in enumerate(((I, H), (I, H), (H, I))):
            ptr, _ = self.tables[p].storage()
            h = C.c_void_p()
            ctx.check(ctx.lib.har_cuda_weights_wrap_q4k(ctx.handle, C.c_void_p(ptr), n_slots, N, K,
                                                        C.byref(h)))
            w = Q4KWeights(ctx, h, n_slots, N, K)
            w.keepalive = self.tables[p]
            views.append(w)
        self.layer = ctx.moe_layer(views[0], views[1], views[2], shared, sh_gate_inp)
        self.slot_of = {}       # expert -> slot
        self.in_flight = []     # slots acquired for the last dispatch
        self.event = None       # that dispatch's completion event
        self.uploads = 0

    def _settle(self):
        """Release the previous dispatch's slots once its event has completed."""
        if self.event is not None:
            self.event.synchronize()
            for sid in self.in_flight:
                for t in self.tables:
                    t.release(sid, self.event)
            self.in_flight = []

    def ffn(self, x, ids: np.ndarray, weights, y, flags: int = 0):
        """moe_ffn for device x / weights / y and host expert ids [T][k]."""
        import torch
        ids = np.asarray(ids, np.int32)
        need = list(dict.fromkeys(int(e) for e in ids.ravel()))
        if len(need) > self.n_slots:
            raise HarCudaError(ERR_GEOMETRY, "slotted layer: more distinct experts than slots")
        self._settle()
        fresh = []
        for e in need:
            if e in self.slot_of:
                continue
            snaps = self.tables[0].snapshot()
            free = [s for s in snaps if s["state"] == SLOT_FREE]
            if not free:
                keep = {self.slot_of[n] for n in need if n in self.slot_of}
                victims = [s for s in snaps if s["state"] == SLOT_READY and s["slot_id"] not in keep]
                v = min(victims, key=lambda s: s["last_use_epoch"])
                for t in self.tables:
                    t.evict(v["slot_id"], self.event)
                del self.slot_of[v["key"][1]]
            sids = [t.reserve(SlotTable.key(self.layer_id, e, p)) for p, t in enumerate(self.tables)]
            assert len(set(sids)) == 1, sids
            for p, t in enumerate(self.tables):
                t.upload(sids[0], self.host[p][e])
            self.slot_of[e] = sids[0]
            fresh.append(sids[0])
            self.uploads += 1
        if fresh:
            self.ctx.synchronize()  # the uploads' events complete
            for sid in fresh:
                for t in self.tables:
                    t.mark_ready(sid)
        for e in need:
            for p, t in enumerate(self.tables):
                t.acquire(SlotTable.key(self.layer_id, e, p))
        self.in_flight = [self.slot_of[e] for e in need]
        remap = np.vectorize(self.slot_of.__getitem__, otypes=[np.int32])(ids) if ids.size else ids
        sid_dev = torch.from_numpy(np.ascontiguousarray(remap, np.int32)).to(x.device)
        self.ctx.moe_ffn(self.layer, x, sid_dev, weights, y, flags)
        self.event = torch.cuda.Event()
        self.event.record()
        self._ids_keep = sid_dev


# ---------------------------------------------------------------------------
# Reference-interface mirror
# ---------------------------------------------------------------------------

class CudaQ4KModel:
    """The serving-seam model of har/crates/har-serve/src/q4k.rs:129-220 with
    its matvec on the GPU (the role VulkanBatchedModel plays,
    har/crates/har-serve/src/vulkan.rs:286-493): one GEMV launch per step for
    the whole batch, weights read once per step."""

    def __init__(self, ctx: Context, blocks: np.ndarray, rows: int, dim: int, embed: np.ndarray,
                 eos: int, act_kind: int = ACT_F32):
        import torch
        if dim % QK_K:
            raise HarCudaError(ERR_GEOMETRY, "dim must be super-block-aligned")
        self.ctx, self.rows, self.dim, self.eos, self.act_kind = ctx, rows, dim, eos, act_kind
        self.w = ctx.upload_q4k(blocks, 1, rows, dim)
        self.embed = np.ascontiguousarray(embed, np.float32).reshape(-1, dim)
        self._torch = torch

    def matvec(self, x: np.ndarray) -> np.ndarray:
        """Q4KModel::matvec for a batch: rows of x [M][dim] -> [M][rows]."""
        torch = self._torch
        x = np.ascontiguousarray(x, np.float32).reshape(-1, self.dim)
        M = x.shape[0]
        dev = torch.device("cuda", self.ctx.device)
        xd = torch.from_numpy(x).to(dev)
        y = torch.empty((M, self.rows), dtype=torch.float32, device=dev)
        if self.act_kind == ACT_Q8K:
            xq = torch.empty((M, self.dim // QK_K * Q8K_BLOCK_BYTES), dtype=torch.uint8, device=dev)
            self.ctx.q8k_quantize(xd, xq)
            self.ctx.q4k_gemv(self.w, 0, xq, ACT_Q8K, M, y)
        else:
            self.ctx.q4k_gemv(self.w, 0, xd, ACT_F32, M, y)
        return y.cpu().numpy()

    def batch_step(self, inputs):
        """BatchStepModel::batch_step: x = h + E[t]; logits = W x; next = x."""
        xs = np.stack([np.asarray(h, np.float32) + self.embed[t] for h, t in inputs])
        logits = self.matvec(xs)
        return [(xs[i], logits[i]) for i in range(len(inputs))]

    def initial_hidden(self):
        return np.zeros(self.dim, np.float32)

    def weight_bytes_per_row(self) -> int:
        return self.rows * (self.dim // QK_K) * Q4K_BLOCK_BYTES


class CudaMoeModel:
    """Per-layer expert tensors on the device with the reference's expert-FFN
    entry points (har-native-qwen35moe.rs:626-689, 979-1048, 1167-1215)."""

    def __init__(self, ctx: Context, layers, E: int, H: int, I: int, k: int, flags: int = 0):
        self.ctx, self.layers, self.E, self.H, self.I, self.k = ctx, layers, E, H, I, k
        self.flags = flags
        import torch
        self._torch = torch

    def _dev(self, a, dtype):
        torch = self._torch
        return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype).to(
            torch.device("cuda", self.ctx.device))

    def expert_matvec(self, w: Q4KWeights, expert: int, x: np.ndarray) -> np.ndarray:
        torch = self._torch
        if x.shape[-1] != w.K:
            raise HarCudaError(ERR_GEOMETRY, f"expert matvec shape mismatch: K={w.K} input={x.shape[-1]}")
        if not 0 <= expert < w.E:
            raise HarCudaError(ERR_ARG, f"expert {expert} exceeds model expert count {w.E}")
        xd = self._dev(x.reshape(1, -1), torch.float32)
        y = torch.empty((1, w.N), dtype=torch.float32, device=xd.device)
        self.ctx.q4k_gemv(w, expert, xd, ACT_F32, 1, y)
        self.ctx.synchronize()
        return y.cpu().numpy()[0]

    def compose_moe_route(self, layer: int, x: np.ndarray, experts, weights) -> np.ndarray:
        if len(experts) != len(weights) or len(experts) != self.k:
            raise HarCudaError(ERR_GEOMETRY, "route geometry is invalid")
        y = self.ctx.moe_ffn_host(self.layers[layer], np.asarray(x, np.float32).reshape(1, -1),
                                  np.asarray(experts, np.int32).reshape(1, -1),
                                  np.asarray(weights, np.float32).reshape(1, -1), self.flags)
        return y[0]

    def routed_moe(self, layer: int, x: np.ndarray, router_logits: np.ndarray = None):
        """routed_moe (har-native-qwen35moe.rs:1167-1215); returns (out, ids,
        weights).  Without router_logits the layer's own f32 router (a layer
        loaded from GGUF) computes them on the device; with them, only the
        softmax + top-k runs on the device before compose_moe_route."""
        torch = self._torch
        if router_logits is None:
            xd = self._dev(np.asarray(x, np.float32).reshape(1, -1), torch.float32)
            ids = torch.empty((1, self.k), dtype=torch.int32, device=xd.device)
            w = torch.empty((1, self.k), dtype=torch.float32, device=xd.device)
            y = torch.empty_like(xd)
            self.ctx.check(self.ctx.lib.har_cuda_routed_moe(
                self.ctx.handle, self.layers[layer].handle, None, _dptr(xd), 1, self.k,
                _dptr(ids), _dptr(w), _dptr(y), self.flags))
            self.ctx.synchronize()
            return y.cpu().numpy()[0], ids.cpu().numpy()[0], w.cpu().numpy()[0]
        lg = self._dev(np.asarray(router_logits, np.float32).reshape(1, -1), torch.float32)
        ids = torch.empty((1, self.k), dtype=torch.int32, device=lg.device)
        w = torch.empty((1, self.k), dtype=torch.float32, device=lg.device)
        self.ctx.route_topk(lg, self.k, ids, w)
        ids_h, w_h = ids.cpu().numpy(), w.cpu().numpy()
        return self.compose_moe_route(layer, x, ids_h[0], w_h[0]), ids_h[0], w_h[0]

    @classmethod
    def from_gguf(cls, ctx: Context, path: str, k: int = None, flags: int = 0):
        """Every block's MoE layer of a GGUF file on the device; k defaults to
        the file's {arch}.expert_used_count."""
        g = Gguf(path)
        arch = g.meta_string("general.architecture") or ""
        blocks = g.meta_u64(f"{arch}.block_count") or 0
        layers = [ctx.moe_layer_from_gguf(g, b) for b in range(blocks)
                  if g.find(f"blk.{b}.ffn_gate_exps.weight") >= 0]
        if not layers:
            raise HarCudaError(ERR_ARG, f"{path}: no MoE layers")
        E, H, I = layers[0].E, layers[0].H, layers[0].I
        if k is None:
            k = g.meta_u64(f"{arch}.expert_used_count") or 8
        m = cls(ctx, layers, E, H, I, k, flags)
        m.gguf = g
        return m


class StepOutcome:
    """One sequence's result of a step (har/crates/har-serve/src/adapter.rs:74-113);
    plain decode steps only: no drafts, consumed_state == next."""

    __slots__ = ("next", "logits", "drafts", "draft_states", "consumed_state")

    def __init__(self, next_state: np.ndarray, logits: np.ndarray):
        self.next = next_state
        self.logits = logits
        self.drafts = []
        self.draft_states = []
        self.consumed_state = next_state


class CudaMoeServingModel:
    """A BatchStepModel (har/crates/har-serve/src/adapter.rs:28-72) over
    har-cuda: the serving seam's contract with the Q4_K MoE stack on the GPU,
    in the role MoEModel plays for the CPU (har/crates/har-serve/src/moe.rs:182-282).

    One step for a batch of (hidden, token): x = hidden + embed[token]; each
    MoE layer routes x with its f32 router on the device and adds its output
    to x (routed_moe + residual, har-native-qwen35moe.rs:1152-1215); logits =
    out · x with the LM head (Q4_K or Q6_K) GEMV.  Every sequence of the batch
    shares each weight read: one routed_moe per layer and one GEMV per step
    for the whole batch.  `next` is the hidden state after the layers (the
    reference's toy MoEModel returns its input state instead; a real model's
    next state is its last layer's output).  A GPU error raises HarCudaError
    (the fail-closed rule of vulkan.rs:18-19); nothing falls back to the CPU.
    """

    def __init__(self, ctx: Context, layers, embed: np.ndarray, out: Q4KWeights, k: int,
                 eos: int, routers=None, flags: int = 0):
        import torch
        self.ctx, self.layers, self.k, self._eos, self.flags = ctx, list(layers), k, eos, flags
        self.out = out
        self.H = out.K
        self.vocab = out.N
        dev = torch.device("cuda", ctx.device)
        self.embed = torch.from_numpy(np.ascontiguousarray(embed, np.float32).reshape(-1, self.H)).to(dev)
        if self.embed.shape[0] != self.vocab:
            raise HarCudaError(ERR_GEOMETRY, "embed must be [vocab][H] with the LM head's vocab")
        self.routers = list(routers) if routers is not None else [None] * len(self.layers)
        if len(self.routers) != len(self.layers):
            raise HarCudaError(ERR_GEOMETRY, "one router (or None: the layer's own) per layer")
        self._torch = torch
        self._dev = dev
        self.last_routes = None  # [(ids [B][k], weights [B][k]) per layer] of the last step
        self.telemetry = {"positions": 0, "expert_reads": 0, "shared_reads": 0}

    def _step_device(self, x):
        torch = self._torch
        B, L = x.shape[0], len(self.layers)
        # every layer routed and applied in one library call
        ids = torch.empty((L, B, self.k), dtype=torch.int32, device=self._dev)
        w = torch.empty((L, B, self.k), dtype=torch.float32, device=self._dev)
        y = torch.empty_like(x)
        self.ctx.routed_moe_stack(self.layers, self.routers, x, self.k, ids, w, y,
                                  self.flags | MOE_ADD_RESIDUAL)
        routes = [(ids[l], w[l]) for l in range(L)]
        x = y
        logits = torch.empty((B, self.vocab), dtype=torch.float32, device=self._dev)
        if self.out.ggml_type == GGML_Q6_K:
            self.ctx.q6k_gemv(self.out, 0, x, B, logits)
        else:
            self.ctx.q4k_gemv(self.out, 0, x, ACT_F32, B, logits)
        return x, logits, routes

    def batch_step(self, inputs):
        """BatchStepModel::batch_step: inputs [(hidden [H], token)] ->
        [StepOutcome], one per input, in order."""
        torch = self._torch
        if not inputs:
            return []
        h = np.stack([np.asarray(hv, np.float32).reshape(self.H) for hv, _ in inputs])
        tok = np.asarray([t for _, t in inputs], np.int64)
        if tok.min() < 0 or tok.max() >= self.vocab:
            raise HarCudaError(ERR_ARG, "token id outside the vocabulary")
        x = torch.from_numpy(h).to(self._dev) + self.embed[torch.from_numpy(tok).to(self._dev)]
        x, logits, routes = self._step_device(x.contiguous())
        self.ctx.synchronize()
        nxt, lg = x.cpu().numpy(), logits.cpu().numpy()
        self.last_routes = [(i.cpu().numpy(), w.cpu().numpy()) for i, w in routes]
        self.telemetry["positions"] += len(inputs)
        self.telemetry["expert_reads"] += sum(len(np.unique(i)) for i, _ in self.last_routes)
        self.telemetry["shared_reads"] += len(self.layers)
        return [StepOutcome(nxt[i], lg[i]) for i in range(len(inputs))]

    def prefill_batch(self, inputs):
        """The trait's default prefill (adapter.rs:42-61): batch_step folded
        one token at a time per sequence."""
        out = []
        for h, tokens in inputs:
            hidden = np.asarray(h, np.float32)
            states, logits = [], []
            for t in tokens:
                o = self.batch_step([(hidden, t)])[0]
                states.append(o.next)
                logits.append(o.logits)
                hidden = o.next
            out.append((states, logits))
        return out

    def initial_hidden(self) -> np.ndarray:
        return np.zeros(self.H, np.float32)

    def eos(self) -> int:
        return self._eos

    def weight_bytes_per_row(self) -> int:
        """Per-token worst case, as MoEModel counts it (moe.rs:274-281): the
        shared expert plus top_k routed experts per layer, plus the LM head."""
        total = self.out.nbytes
        for layer in self.layers:
            total += (self.k + (1 if layer.shared else 0)) * layer.expert_bytes()
        return total
