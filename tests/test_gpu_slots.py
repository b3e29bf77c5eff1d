"""Expert-slot residency on the GPU: projections uploaded into a slot table's
device storage are what the kernels read, and a layer served from a few slots
(experts uploaded on demand, least recently used slots evicted) gives the
fully resident layer's results bit for bit."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import haro  # noqa: E402
import har_cuda  # noqa: E402
from har_cuda import SlotTable, SlottedMoeLayer, PROJ_GATE, SLOT_IN_FLIGHT, SLOT_READY  # noqa: E402
from gpu_util import Layer, to_dev  # noqa: E402

E, H, I, K = 32, 2048, 512, 4


@pytest.fixture(scope="module")
def ctx():
    c = har_cuda.Context(0)
    yield c
    torch.cuda.synchronize()
    c.close()


@pytest.fixture(scope="module")
def layer(ctx):
    return Layer(ctx, E, H, I, seed=7300)


def test_upload_lands_in_its_slot(ctx, layer):
    pb = I * (H // 256) * 144
    t = SlotTable(ctx, 4, pb)
    sid = t.reserve(t.key(0, 3, PROJ_GATE))
    t.upload(sid, layer.hg.reshape(E, pb)[3])
    ctx.synchronize()
    t.mark_ready(sid)
    ptr, nbytes = t.storage()
    assert nbytes == 4 * pb
    h = ctypes.c_void_p()
    ctx.check(ctx.lib.har_cuda_weights_wrap_q4k(ctx.handle, ctypes.c_void_p(ptr), 4, I, H, ctypes.byref(h)))
    w = har_cuda.Q4KWeights(ctx, h, 4, I, H)
    x = haro.normal_f32(7301, 0, H).reshape(1, H)
    y = torch.empty((1, I), dtype=torch.float32, device="cuda")
    ctx.q4k_gemv(w, sid, to_dev(x), har_cuda.ACT_F32, 1, y)
    torch.cuda.synchronize()
    ref = haro.expert_matvec(layer.hg, E, I, H, 3, x[0])
    assert np.allclose(y.cpu().numpy()[0], ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())
    # a complete event releases / evicts; the slot's record follows the rules
    got = t.acquire(t.key(0, 3, PROJ_GATE))
    assert got["state"] == SLOT_IN_FLIGHT
    ev = torch.cuda.Event()
    ev.record()
    ev.synchronize()
    t.release(sid, ev)
    assert t.snapshot()[sid]["state"] == SLOT_READY
    t.evict(sid, ev)
    t.free()


@pytest.mark.parametrize("flags", [0, har_cuda.MOE_DECODE])
def test_slotted_layer_equals_resident_layer(ctx, layer, flags):
    # 8 slots for 32 experts; each call needs at most 8 (2 tokens x top-4)
    sl = SlottedMoeLayer(ctx, layer.hg, layer.hu, layer.hd, E, H, I, n_slots=8,
                         shared=layer.weights[3], sh_gate_inp=layer.gi_dev)
    distinct = set()
    for call in range(6):
        x = haro.normal_f32(7310 + call, 0, 2 * H).reshape(2, H)
        ids, w = haro.route_topk(haro.normal_f32(7320 + call, 0, 2 * E).reshape(2, E), K)
        distinct |= set(ids.ravel().tolist())
        xd, wd = to_dev(x), to_dev(w)
        ys = torch.empty_like(xd)
        sl.ffn(xd, ids, wd, ys, flags)
        yr = torch.empty_like(xd)
        ctx.moe_ffn(layer.layer, xd, to_dev(ids), wd, yr, flags)
        torch.cuda.synchronize()
        ctx.synchronize()
        assert np.array_equal(ys.cpu().numpy(), yr.cpu().numpy()), call
    assert len(distinct) > 8 and sl.uploads >= len(distinct)   # slots were evicted and refilled
    states = [s["state"] for s in sl.tables[0].snapshot()]
    assert states.count(SLOT_IN_FLIGHT) == len(sl.in_flight)     # the last dispatch's slots
