"""The serving seam over har-cuda: CudaMoeServingModel, a BatchStepModel
(har/crates/har-serve/src/adapter.rs:28-72) whose step is the MoE stack with
device routing plus an LM-head GEMV, loaded from a GGUF file, against the
CPU restatement of the same step; batched equals isolated
(har/crates/har-serve/src/moe.rs:301-314)."""
import numpy as np
import pytest

import har_cuda
import haro
from _common import assert_close
from gguf_writer import STRING, U32, write_gguf
from test_gguf import GT_F32, GT_Q4K, GT_Q6K, _moe_file

pytestmark = pytest.mark.gpu

E, H, I, V, K_USED = 8, 512, 256, 300, 4


@pytest.fixture(scope="module")
def served(tmp_path_factory):
    p = tmp_path_factory.mktemp("serve") / "m.gguf"
    host = _moe_file(p, E, H, I, 1200, layers=2)
    # append the embedding and LM head by rewriting the file with them
    tensors = []
    for b in range(2):
        hg, hu, hd, (sg, su, sd), gi, rt = host[b]
        q = f"blk.{b}."
        tensors += [(q + "ffn_gate_exps.weight", [H, I, E], GT_Q4K, hg),
                    (q + "ffn_up_exps.weight", [H, I, E], GT_Q4K, hu),
                    (q + "ffn_down_exps.weight", [I, H, E], GT_Q4K, hd),
                    (q + "ffn_gate_shexp.weight", [H, I], GT_Q4K, sg),
                    (q + "ffn_up_shexp.weight", [H, I], GT_Q4K, su),
                    (q + "ffn_down_shexp.weight", [I, H], GT_Q4K, sd),
                    (q + "ffn_gate_inp_shexp.weight", [H], GT_F32, gi),
                    (q + "ffn_gate_inp.weight", [H, E], GT_F32, rt)]
    embed = haro.normal_f32(1300, 0, V * H, 0.0, 0.5).reshape(V, H)
    out = haro.random_q6k(1301, V, H)
    tensors += [("token_embd.weight", [H, V], GT_F32, embed), ("output.weight", [H, V], GT_Q6K, out)]
    write_gguf(p, [("general.architecture", STRING, "qwen35moe"),
                   ("qwen35moe.block_count", U32, 2), ("qwen35moe.expert_count", U32, E),
                   ("qwen35moe.expert_used_count", U32, K_USED)], tensors)
    ctx = har_cuda.Context(0)
    moe = har_cuda.CudaMoeModel.from_gguf(ctx, str(p))
    head = ctx.weights_from_gguf(moe.gguf, "output.weight")
    yield ctx, moe, head, host, embed, out
    ctx.close()


def _oracle_step(host, embed, out, h, t):
    x = (h + embed[t]).astype(np.float32).reshape(1, H)
    routes = []
    for b in range(2):
        hg, hu, hd, sh, gi, rt = host[b]
        ids, w = haro.route_topk(haro.router_logits(rt, x), K_USED, exp_mode=0)
        routes.append(ids[0])
        x = haro.moe_ffn(hg, hu, hd, sh, gi, E, H, I, x, ids, w, add_residual=True)
    return x[0], haro.q6k_matvec(out, V, H, x)[0], routes


def test_batch_step_matches_oracle(served):
    ctx, moe, head, host, embed, out = served
    model = har_cuda.CudaMoeServingModel(ctx, moe.layers, embed, head, K_USED, eos=V - 1,
                                         flags=har_cuda.MOE_FORCE_GEMV)
    hs = [haro.normal_f32(1400 + i, 0, H, 0.0, 0.3) for i in range(3)]
    toks = [5, 77, 299]
    outs = model.batch_step(list(zip(hs, toks)))
    assert len(outs) == 3
    for i in range(3):
        nxt, lg, routes = _oracle_step(host, embed, out, hs[i], toks[i])
        for b in range(2):
            assert np.array_equal(model.last_routes[b][0][i], routes[b]), (i, b)
        assert_close(outs[i].next, nxt, what=f"next {i}")
        assert_close(outs[i].logits, lg, what=f"logits {i}")
        assert outs[i].drafts == [] and outs[i].consumed_state is outs[i].next
    assert model.telemetry["positions"] == 3
    assert model.eos() == V - 1
    assert np.array_equal(model.initial_hidden(), np.zeros(H, np.float32))
    per = 3 * I * (H // 256) * 144
    assert model.weight_bytes_per_row() == head.nbytes + 2 * (K_USED + 1) * per


def test_batched_equals_isolated_and_prefill(served):
    """The tensor-core default path: a sequence's step does not depend on
    the other sequences of the batch (moe.rs:301-314)."""
    ctx, moe, head, host, embed, out = served
    model = har_cuda.CudaMoeServingModel(ctx, moe.layers, embed, head, K_USED, eos=V - 1)
    hs = [haro.normal_f32(1500 + i, 0, H, 0.0, 0.3) for i in range(4)]
    toks = [1, 2, 150, 7]
    batched = model.batch_step(list(zip(hs, toks)))
    for i in range(4):
        alone = model.batch_step([(hs[i], toks[i])])[0]
        assert np.array_equal(alone.next, batched[i].next), i
        assert_close(alone.logits, batched[i].logits, rel=1e-6, what=f"logits {i}")
    # prefill folds batch_step token by token (adapter.rs:42-61)
    (states, logits), = model.prefill_batch([(hs[0], [3, 9])])
    a = model.batch_step([(hs[0], 3)])[0]
    b = model.batch_step([(a.next, 9)])[0]
    assert np.array_equal(states[0], a.next) and np.array_equal(states[1], b.next)
    assert np.array_equal(logits[1], b.logits)
    with pytest.raises(har_cuda.HarCudaError):
        model.batch_step([(hs[0], V)])                     # token outside the vocabulary


@pytest.mark.parametrize("flags", [0, har_cuda.MOE_FORCE_GEMV])
def test_routed_stack_equals_per_layer_calls(served, flags):
    """har_cuda_routed_moe_stack (every layer routed on the device in one call)
    equals routed_moe called layer by layer, bit for bit, route records
    included; input and output may alias."""
    import torch

    ctx, moe, head, host, embed, out = served
    T, k = 5, K_USED
    x = torch.from_numpy(haro.normal_f32(1600, 0, T * H, 0.0, 0.5).reshape(T, H)).cuda()
    f = flags | har_cuda.MOE_ADD_RESIDUAL
    ids = torch.empty((2, T, k), dtype=torch.int32, device="cuda")
    w = torch.empty((2, T, k), dtype=torch.float32, device="cuda")
    y = torch.empty_like(x)
    ctx.routed_moe_stack(moe.layers, None, x, k, ids, w, y, f)
    cur = x.clone()
    for l in range(2):
        i1 = torch.empty((T, k), dtype=torch.int32, device="cuda")
        w1 = torch.empty((T, k), dtype=torch.float32, device="cuda")
        nxt = torch.empty_like(cur)
        ctx.routed_moe(moe.layers[l], None, cur, k, i1, w1, nxt, f)
        assert torch.equal(i1, ids[l]) and torch.equal(w1, w[l])
        cur = nxt
    ctx.synchronize()
    assert torch.equal(cur, y)
    xa = x.clone()                                   # aliased input and output
    ctx.routed_moe_stack(moe.layers, [None, None], xa, k, ids, w, xa, f)
    ctx.synchronize()
    assert torch.equal(xa, y)
