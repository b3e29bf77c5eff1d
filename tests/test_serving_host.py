"""Host logic of the serving adapter (har_cuda.CudaMoeServingModel) on the CPU:
the default prefill folds batch_step one token at a time
(har/crates/har-serve/src/adapter.rs:42-61), a step outcome is a plain decode
step (adapter.rs:103-113), and the per-row weight accounting counts top_k
routed experts plus the shared expert per layer (moe.rs:274-281) at the
Alice expert size of 1,769,472 bytes.  The device step itself is covered by
tests/test_gpu_serving.py."""
import numpy as np

import har_cuda


class _NumpyStep(har_cuda.CudaMoeServingModel):
    """The adapter with its device step replaced by a numpy rule."""

    def __init__(self, H, V):  # no device state
        self.H, self.vocab, self._eos = H, V, V - 1
        self.calls = []

    def batch_step(self, inputs):
        self.calls.append(len(inputs))
        return [har_cuda.StepOutcome(np.asarray(h, np.float32) * 0.5 + t,
                                     np.full(self.vocab, t, np.float32)) for h, t in inputs]


def test_prefill_folds_batch_step_token_by_token():
    m = _NumpyStep(4, 10)
    (states, logits), (states2, _) = m.prefill_batch([(np.ones(4, np.float32), [3, 7]),
                                                      (np.zeros(4, np.float32), [1])])
    assert np.allclose(states[0], 3.5) and np.allclose(states[1], 3.5 * 0.5 + 7)
    assert logits[0][0] == 3 and logits[1][0] == 7
    assert np.allclose(states2[0], 1.0)
    assert m.calls == [1, 1, 1]                 # one single-sequence step per token
    assert m.eos() == 9 and np.array_equal(m.initial_hidden(), np.zeros(4, np.float32))


def test_step_outcome_is_a_plain_decode_step():
    o = har_cuda.StepOutcome(np.ones(3, np.float32), np.zeros(5, np.float32))
    assert o.drafts == [] and o.draft_states == [] and o.consumed_state is o.next


def test_weight_bytes_per_row_alice_layers():
    m = object.__new__(har_cuda.CudaMoeServingModel)
    m.k = 10
    m.out = type("Head", (), {"nbytes": 4096})()
    layer = object.__new__(har_cuda.MoeLayer)
    layer.handle = None
    layer.E, layer.H, layer.I, layer.shared = 512, 2048, 512, True
    assert layer.expert_bytes() == 1_769_472
    m.layers = [layer] * 48
    assert m.weight_bytes_per_row() == 4096 + 48 * 11 * 1_769_472
    layer.shared = False
    assert m.weight_bytes_per_row() == 4096 + 48 * 10 * 1_769_472
