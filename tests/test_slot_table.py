"""The expert-slot table's state machine (ExpertSlotTable,
har/crates/har-vulkan/src/lib.rs:1233-1460) through the C ABI, on a table
without storage (no GPU): every transition rule and error case of the
reference, and the epochs it stamps."""
import pytest

import har_cuda
from har_cuda import SlotTable, PROJ_GATE, PROJ_UP, PROJ_DOWN, SLOT_FREE, SLOT_UPLOADING, SLOT_READY, SLOT_IN_FLIGHT


def err(fn, *a):
    with pytest.raises(har_cuda.HarCudaError) as e:
        fn(*a)
    return str(e.value)


def test_create_checks_dimensions():
    # create_expert_slot_table (lib.rs:930-936)
    for count, nbytes in ((0, 4096), (2, 0), (2, 1 << 63)):
        with pytest.raises(har_cuda.HarCudaError) as e:
            SlotTable(None, count, nbytes)
        assert e.value.status == har_cuda.ERR_ARG
    t = SlotTable(None, 2, 4096)
    assert t.storage() == (0, 8192)   # no storage without a context; the size is count x bytes
    snaps = t.snapshot()
    assert [s["slot_id"] for s in snaps] == [0, 1]
    assert all(s["state"] == SLOT_FREE and not s["ready"] and s["last_use_epoch"] == 0 for s in snaps)


def test_life_cycle_and_epochs():
    t = SlotTable(None, 2, 4096)
    a, b, c = t.key(3, 7, PROJ_GATE), t.key(3, 7, PROJ_UP), t.key(3, 9, PROJ_DOWN)
    assert t.reserve(a) == 0                                   # the first Free slot
    s0 = t.snapshot()[0]
    assert (s0["state"], s0["upload_epoch"], s0["last_use_epoch"]) == (SLOT_UPLOADING, 1, 1)
    assert "already resident or in flight" in err(t.reserve, a)
    assert "generation zero is reserved" in err(t.reserve, t.key(3, 7, PROJ_GATE, 0))
    assert t.reserve(b) == 1
    assert "bounded slot table is full" in err(t.reserve, c)
    # mark_ready needs a submitted upload (lib.rs:1353-1357)
    assert "no submitted upload event" in err(t.mark_ready, 0)
    t.mark_upload_submitted(0)
    assert "slot is not ready" in err(t.acquire, b)            # b is still uploading
    t.mark_ready(0)
    s0 = t.snapshot()[0]
    assert s0["state"] == SLOT_READY and s0["ready"]
    assert "slot is not uploading" in err(t.mark_ready, 0)
    assert "not awaiting upload" in err(t.mark_upload_submitted, 0)
    got = t.acquire(a)                                          # epoch 3 (1, 2 went to reserves)
    assert got["slot_id"] == 0 and got["state"] == SLOT_IN_FLIGHT and got["last_use_epoch"] == 3
    assert "cannot evict an in-flight slot" in err(t.evict, 0)
    t.release(0)
    s0 = t.snapshot()[0]
    assert s0["state"] == SLOT_READY and s0["last_use_epoch"] == 4
    assert "slot is not in flight" in err(t.release, 0)
    t.evict(0)                                                  # Ready slots may go
    s0 = t.snapshot()[0]
    assert s0["state"] == SLOT_FREE and s0["key"] == (0, 0, 0, 0) and s0["last_use_epoch"] == 5
    assert "not resident" in err(t.acquire, a)
    assert t.reserve(c) == 0                                    # the freed slot is reused
    t.evict(1)                                                  # an Uploading slot may go too
    assert t.snapshot()[1]["state"] == SLOT_FREE


def test_slot_ids_and_events_are_checked():
    t = SlotTable(None, 1, 64)
    for fn in (t.mark_upload_submitted, t.mark_ready, t.release, t.evict):
        assert "outside table" in err(fn, 5)
    k = t.key(0, 1, PROJ_GATE)
    t.reserve(k)
    # a table without storage takes only NULL events ("already complete")
    assert "without storage" in err(t.mark_upload_submitted, 0, 0x1234)
    assert "without storage" in err(t.release, 0, 0x1234)
    # the library's own upload needs storage
    import numpy as np
    assert "no storage" in err(t.upload, 0, np.zeros(16, np.uint8))
