"""GGUF expert loader (include/har_cuda.h har_cuda_gguf_*): the directory
parse against files written to the format (host-only, no GPU), its error
handling, and on the GPU the upload of expert, shared-expert, router, Q6_K and Q3_K
tensors checked through the kernels against the oracle.

The parse follows GgufReader::inspect (har/crates/har-model/src/lib.rs:126-399);
the geometry known answer is the reference's own (lib.rs:653-657: a Q4_K
tensor of 5,120 values has a 2,880-byte payload)."""
import struct

import numpy as np
import pytest

import har_cuda
import haro
from gguf_writer import (ARRAY, BOOL, F32, I64, STRING, U32, U64, write_gguf)

GT_F32, GT_Q3K, GT_Q4K, GT_Q6K = 0, 11, 12, 14


def _meta(extra=()):
    return [("general.architecture", STRING, "qwen35moe"),
            ("general.name", STRING, "tiny-moe"),
            ("general.alignment", U32, 64),
            ("qwen35moe.block_count", U32, 2),
            ("qwen35moe.expert_count", U64, 4),
            ("qwen35moe.expert_used_count", U32, 2),
            ("qwen35moe.rope.freq_base", F32, 10000.0),
            ("qwen35moe.some_flag", BOOL, True),
            ("qwen35moe.signed", I64, -5),
            ("tokenizer.ggml.tokens", ARRAY, (STRING, ["<s>", "</s>", "hello"])),
            ("tokenizer.ggml.scores", ARRAY, (F32, [0.0, -1.0, -2.5])),
            ("nested", ARRAY, (ARRAY, [(U32, [1, 2]), (U32, [3])]))] + list(extra)


def test_parse_directory(tmp_path):
    E, H, I = 4, 512, 256
    gate = np.arange(E * I * (H // 256) * 144, dtype=np.uint32).astype(np.uint8)
    q6 = haro.random_q6k(5, 16, 256)
    router = np.arange(E * H, dtype=np.float32)
    odd = np.arange(70, dtype=np.uint8)            # type not in the tables
    tensors = [("blk.0.ffn_gate_exps.weight", [H, I, E], GT_Q4K, gate),
               ("output.weight", [256, 16], GT_Q6K, q6),
               ("blk.0.ffn_gate_inp.weight", [H, E], GT_F32, router),
               ("weird.weight", [70], 99, odd)]
    p = tmp_path / "t.gguf"
    where = write_gguf(p, _meta(), tensors, alignment=64)
    g = har_cuda.Gguf(str(p))
    assert (g.version, g.tensor_count, g.metadata_count, g.alignment) == (3, 4, 12, 64)
    assert g.data_offset % 64 == 0
    infos = g.tensors()
    for info, (name, dims, gt, payload) in zip(infos, tensors):
        assert info["name"] == name and info["dims"] == dims and info["type"] == gt
        assert info["file_offset"] == where[name]
    assert infos[0]["payload_bytes"] == gate.size
    assert infos[1]["payload_bytes"] == 16 * 210
    assert infos[2]["payload_bytes"] == E * H * 4
    # unknown type: the span to the end of the file
    assert infos[3]["payload_bytes"] == p.stat().st_size - where["weird.weight"]
    assert g.find("output.weight") == 1 and g.find("missing") == -1
    assert g.meta_u64("qwen35moe.expert_count") == 4
    assert g.meta_u64("qwen35moe.block_count") == 2
    assert g.meta_u64("qwen35moe.rope.freq_base") == 10000    # integral float, as "10000"
    assert g.meta_u64("qwen35moe.signed") is None
    assert g.meta_u64("qwen35moe.some_flag") is None
    assert g.meta_string("general.architecture") == "qwen35moe"
    assert g.meta_string("qwen35moe.expert_count") is None
    # the bytes at the reported offset are the tensor's
    raw = p.read_bytes()
    off = infos[1]["file_offset"]
    assert raw[off:off + 16 * 210] == q6.tobytes()
    g.close()


def test_reference_q4k_geometry_known_answer(tmp_path):
    """har/crates/har-model/src/lib.rs:653-657: tensor_payload_bytes(12, 5120) == 2880."""
    p = tmp_path / "g.gguf"
    write_gguf(p, [], [("blk.0.ffn_gate.weight", [5120, 1], GT_Q4K,
                        np.zeros(2880, np.uint8))])
    g = har_cuda.Gguf(str(p))
    assert g.alignment == 32                                   # the default
    assert g.tensor_info(0)["payload_bytes"] == 2880
    g.close()


def _header(version=3, tensors=0, kv=0):
    return b"GGUF" + struct.pack("<IQQ", version, tensors, kv)


@pytest.mark.parametrize("blob,code", [
    (b"GGUX" + b"\0" * 20, har_cuda.ERR_GEOMETRY),                     # bad magic
    (_header(version=4), har_cuda.ERR_UNSUPPORTED),                   # version 4
    (_header(version=0), har_cuda.ERR_UNSUPPORTED),
    (b"GGUF\x03\0", har_cuda.ERR_GEOMETRY),                            # truncated header
    (_header(tensors=10_000_001), har_cuda.ERR_GEOMETRY),             # count bound
    (_header(kv=1) + struct.pack("<Q", 2**30 + 1), har_cuda.ERR_GEOMETRY),   # string bound
    (_header(kv=1) + struct.pack("<Q", 1) + b"k" + struct.pack("<IIQ", 9, 4, 1_000_001),
     har_cuda.ERR_GEOMETRY),                                           # array bound
    (_header(kv=1) + struct.pack("<Q", 1) + b"k" + struct.pack("<I", 13),
     har_cuda.ERR_GEOMETRY),                                           # unknown value type
    (_header(tensors=1) + struct.pack("<Q", 1) + b"t" + struct.pack("<I", 17),
     har_cuda.ERR_GEOMETRY),                                           # rank 17
    (_header(kv=1) + struct.pack("<Q", 1) + b"k" + struct.pack("<I", 8) + struct.pack("<Q", 50),
     har_cuda.ERR_GEOMETRY),                                           # string past the end
    (_header(tensors=1) + struct.pack("<Q", 1) + b"t" + struct.pack("<IQQIQ", 2, 2**40, 2**40, 0, 0),
     har_cuda.ERR_GEOMETRY),                                           # element count overflows
])
def test_malformed_files_fail_closed(tmp_path, blob, code):
    p = tmp_path / "bad.gguf"
    p.write_bytes(blob)
    with pytest.raises(har_cuda.HarCudaError) as e:
        har_cuda.Gguf(str(p))
    assert e.value.status == code


def test_missing_file(tmp_path):
    with pytest.raises(har_cuda.HarCudaError) as e:
        har_cuda.Gguf(str(tmp_path / "nope.gguf"))
    assert e.value.status == har_cuda.ERR_ARG


def _moe_file(path, E, H, I, seed, layers=1, router=True):
    """An Alice-shaped (small) MoE GGUF: per block the three expert tensors,
    the shared expert, its gate row and the f32 router."""
    host = {}
    tensors = []
    for b in range(layers):
        s = seed + 10 * b
        hg = haro.gen_q4k(s + 1, E * I, H)
        hu = haro.gen_q4k(s + 2, E * I, H)
        hd = haro.gen_q4k(s + 3, E * H, I)
        sg, su, sd = haro.gen_q4k(s + 4, I, H), haro.gen_q4k(s + 5, I, H), haro.gen_q4k(s + 6, H, I)
        gi = haro.normal_f32(s + 7, 0, H, 0.0, 0.02)
        rt = haro.normal_f32(s + 8, 0, E * H, 0.0, 0.02).reshape(E, H)
        p = f"blk.{b}."
        tensors += [(p + "ffn_gate_exps.weight", [H, I, E], GT_Q4K, hg),
                    (p + "ffn_up_exps.weight", [H, I, E], GT_Q4K, hu),
                    (p + "ffn_down_exps.weight", [I, H, E], GT_Q4K, hd),
                    (p + "ffn_gate_shexp.weight", [H, I], GT_Q4K, sg),
                    (p + "ffn_up_shexp.weight", [H, I], GT_Q4K, su),
                    (p + "ffn_down_shexp.weight", [I, H], GT_Q4K, sd),
                    (p + "ffn_gate_inp_shexp.weight", [H], GT_F32, gi)]
        if router:
            tensors.append((p + "ffn_gate_inp.weight", [H, E], GT_F32, rt))
        host[b] = (hg, hu, hd, (sg, su, sd), gi, rt)
    meta = [("general.architecture", STRING, "qwen35moe"),
            ("qwen35moe.block_count", U32, layers),
            ("qwen35moe.expert_count", U32, E),
            ("qwen35moe.expert_used_count", U32, 4)]
    write_gguf(path, meta, tensors)
    return host


@pytest.mark.gpu
def test_moe_model_from_gguf_routes_and_matches_oracle(tmp_path):
    """routed_moe of layers loaded from a GGUF file: the device router's
    record bit-exact, the output within the layer tolerances."""
    from _common import TC_NRMS, assert_close

    ctx = har_cuda.Context(0)
    E, H, I, T = 8, 512, 256, 3
    p = tmp_path / "moe.gguf"
    host = _moe_file(p, E, H, I, 700, layers=2)
    model = har_cuda.CudaMoeModel.from_gguf(ctx, str(p))
    assert (model.E, model.H, model.I, model.k, len(model.layers)) == (E, H, I, 4, 2)
    for layer in range(2):
        hg, hu, hd, sh, gi, rt = host[layer]
        for t in range(T):
            x = haro.normal_f32(800 + 10 * layer + t, 0, H)
            y, ids, w = model.routed_moe(layer, x)
            ref_ids, ref_w = haro.route_topk(haro.router_logits(rt, x.reshape(1, H)), 4, exp_mode=0)
            assert np.array_equal(ids, ref_ids[0])
            assert np.array_equal(w.view(np.uint32), ref_w[0].view(np.uint32))
            ref = haro.moe_ffn(hg, hu, hd, sh, gi, E, H, I, x.reshape(1, H), ref_ids, ref_w)
            assert_close(y.reshape(1, H), ref, nrms=TC_NRMS, what=f"gguf layer {layer} t {t}")
    ctx.close()


@pytest.mark.gpu
def test_weights_from_gguf_q4k_q6k_q3k_and_f32(tmp_path):
    import torch
    from _common import assert_close

    ctx = har_cuda.Context(0)
    E, N, K = 3, 40, 512
    q4 = haro.gen_q4k(901, E * N, K)
    q6 = haro.random_q6k(902, N, K)
    q3 = haro.random_q3k(905, N, K)
    f = haro.normal_f32(903, 0, 5 * 7)
    p = tmp_path / "w.gguf"
    write_gguf(p, [], [("a.weight", [K, N, E], GT_Q4K, q4),
                       ("b.weight", [K, N], GT_Q6K, q6),
                       ("c.weight", [7, 5], GT_F32, f),
                       ("d.weight", [K, N], GT_Q3K, q3)])
    g = har_cuda.Gguf(str(p))
    w4 = ctx.weights_from_gguf(g, "a.weight")
    w6 = ctx.weights_from_gguf(g, "b.weight")
    assert (w4.E, w4.N, w4.K, w6.E, w6.ggml_type) == (E, N, K, 1, GT_Q6K)
    x = haro.normal_f32(904, 0, 2 * K).reshape(2, K)
    xd = torch.from_numpy(x).cuda()
    y = torch.empty((2, N), dtype=torch.float32, device="cuda")
    for e in range(E):
        ctx.q4k_gemv(w4, e, xd, har_cuda.ACT_F32, 2, y)
        torch.cuda.synchronize()
        ref = np.stack([haro.q4k_matvec(q4[e * N:(e + 1) * N], N, K, x[m]) for m in range(2)])
        assert_close(y.cpu().numpy(), ref, what=f"gguf q4k expert {e}")
    ctx.q6k_gemv(w6, 0, xd, 2, y)
    torch.cuda.synchronize()
    assert_close(y.cpu().numpy(), haro.q6k_matvec(q6, N, K, x), what="gguf q6k")
    w3 = ctx.weights_from_gguf(g, "d.weight")
    assert (w3.E, w3.N, w3.K, w3.ggml_type) == (1, N, K, GT_Q3K)
    ctx.q3k_gemv(w3, 0, xd, 2, y)
    torch.cuda.synchronize()
    assert_close(y.cpu().numpy(), haro.q3k_matvec(q3, N, K, x), what="gguf q3k")
    w3.free()
    fd = torch.empty(35, dtype=torch.float32, device="cuda")
    ctx.gguf_read_f32(g, "c.weight", fd)
    torch.cuda.synchronize()
    assert np.array_equal(fd.cpu().numpy(), f)
    with pytest.raises(har_cuda.HarCudaError) as e:
        ctx.weights_from_gguf(g, "c.weight")                     # F32 is not a block type
    assert e.value.status == har_cuda.ERR_UNSUPPORTED
    with pytest.raises(har_cuda.HarCudaError):
        ctx.gguf_read_f32(g, "c.weight", torch.empty(34, dtype=torch.float32, device="cuda"))
    w4.free()
    w6.free()
    g.close()
    ctx.close()


class _DeviceBytes:
    """A view of n device bytes at ptr, for torch.as_tensor (only read here)."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3}


@pytest.mark.gpu
def test_large_tensor_streams_through_both_stages_byte_exact(tmp_path):
    """A tensor larger than one 64 MiB staging buffer arrives in pieces that
    alternate between the two pinned buffers (an Alice `*_exps` tensor is
    302 MB); the device copy equals the file's bytes exactly."""
    import torch

    ctx = har_cuda.Context(0)
    E, N, K = 160, 512, 2048                      # 160 x 589,824 B = 94.4 MB: two pieces
    nbytes = E * N * (K // 256) * 144
    payload = np.random.default_rng(5).integers(0, 256, nbytes, dtype=np.uint8)
    p = tmp_path / "big.gguf"
    write_gguf(p, [], [("blk.0.ffn_up_exps.weight", [K, N, E], GT_Q4K, payload)])
    g = har_cuda.Gguf(str(p))
    w = ctx.weights_from_gguf(g, "blk.0.ffn_up_exps.weight")
    torch.cuda.synchronize()
    ptr = ctx.lib.har_cuda_weights_device_ptr(w.handle)
    got = torch.as_tensor(_DeviceBytes(ptr, nbytes), device="cuda").cpu().numpy()
    assert np.array_equal(got, payload)
    w.free()
    g.close()
    ctx.close()


def test_version_1_and_string_alignment(tmp_path):
    """read_directory accepts versions 1..3 (har-model/src/lib.rs:325-331), and
    metadata_number parses a value's text (:541-543), so an alignment stored as
    the string "64" counts; a negative one falls back to 32."""
    payload = np.zeros(144, np.uint8)
    p = tmp_path / "v1.gguf"
    where = write_gguf(p, [("general.alignment", STRING, "64")],
                       [("t.weight", [256, 1], GT_Q4K, payload)], alignment=64, version=1)
    g = har_cuda.Gguf(str(p))
    assert g.version == 1 and g.alignment == 64 and g.data_offset % 64 == 0
    assert g.tensor_info(0)["file_offset"] == where["t.weight"]
    g.close()
    from gguf_writer import I32
    q = tmp_path / "neg.gguf"
    write_gguf(q, [("general.alignment", I32, -8)], [("t.weight", [256, 1], GT_Q4K, payload)])
    g = har_cuda.Gguf(str(q))
    assert g.alignment == 32
    g.close()
