"""Expert record store and slot window on CPU (open_rknpu2_lm_infer_b200.experts).

Ports the reference's tests of src/model/experts/store.rs:296-317,433-478 and
src/model/experts/window.rs:119-157.
"""
import os

import pytest

from open_rknpu2_lm_infer_b200.experts import (PAGE, Geometry, Store, StoreError, Window, Writer,
                                               lock, tail_experts)


def _geometry(experts=2):
    return Geometry(native_version=1, layers=1, experts=experts, hidden=64, intermediate=64,
                    down_bits=4)


def test_positional_records_are_page_aligned_and_partial_files_are_rejected(tmp_path):
    g = _geometry()
    w = Writer(tmp_path, g, [], 7936)
    w.write(0, 0, bytes([17]) * 7936)
    w.write(0, 1, bytes([29]) * 7936)
    w.finish()
    store = Store(tmp_path, g, [])
    newer = Geometry(**{**g.__dict__, "native_version": 2})
    with pytest.raises(StoreError, match="format v1 requires rebuilding for v2"):
        Store(tmp_path, newer, [])
    repacked = Geometry(**{**g.__dict__, "packing_revision": 1})
    with pytest.raises(StoreError, match="packing revision 0 requires rebuilding for 1"):
        Store(tmp_path, repacked, [])
    assert bytes(store.read(0, 1).as_bytes()) == bytes([29]) * 7936
    assert bytes(store.read(0, 0).as_bytes()) == bytes([17]) * 7936
    batch = store.read_batch(0, 0, 2)
    assert bytes(batch[0].as_bytes()) == bytes([17]) * 7936
    assert bytes(batch[1].as_bytes()) == bytes([29]) * 7936
    with pytest.raises(StoreError):
        store.read(1, 0)
    store.close()
    os.truncate(tmp_path / "experts.npu", 4096)
    with pytest.raises(StoreError):
        Store(tmp_path, g, [])


def test_returned_buffers_are_overwritten_before_reuse(tmp_path):
    g = _geometry(3)
    w = Writer(tmp_path, g, [], PAGE)
    for e in range(3):
        w.write(0, e, bytes([e]) * PAGE)
    w.finish()
    store = Store(tmp_path, g, [])
    for e in (2, 0, 1, 2):
        rec = store.read(0, e)
        assert rec.address() % PAGE == 0
        assert bytes(rec.as_bytes()) == bytes([e]) * PAGE
        rec.release()
    assert store.buffer_stats()["allocations"] == 1
    assert store.buffer_stats()["reuses"] == 3
    records = store.read_batch(0, 0, 3)
    for e, rec in enumerate(records):
        assert bytes(rec.as_bytes()) == bytes([e]) * PAGE
    assert store.buffer_stats()["allocations"] == 3
    for rec in records:
        rec.release()
    assert store.buffer_stats()["idle_buffers"] == 3


def test_writer_rejects_out_of_order_and_missing_records(tmp_path):
    g = _geometry()
    w = Writer(tmp_path, g, [("config.json", 2, 3)], 100)
    with pytest.raises(StoreError):
        w.write(0, 1, bytes(100))
    with pytest.raises(StoreError):
        w.write(0, 0, bytes(99))
    w.write(0, 0, bytes(100))
    with pytest.raises(StoreError, match="missing"):
        w.finish()
    # sources are part of the identity of a cache
    w.write(0, 1, bytes(100))
    w.finish()
    Store(tmp_path, g, [("config.json", 2, 3)]).close()
    with pytest.raises(StoreError, match="does not match"):
        Store(tmp_path, g, [("config.json", 2, 4)])
    with lock(tmp_path) as fh:
        assert fh is not None


def test_pending_imports_do_not_publish_or_evict_requested_weights():
    w = Window(3)
    w.publish(0, 4)
    w.publish(1, 5)
    w.publish(2, 6)
    assert w.plan([4, 7, 8]) == [(7, 1), (8, 2)]
    assert w.slot(4) == 0 and w.slot(7) is None and w.slot(5) == 1


def test_predictions_protect_lru_entries_with_a_fallback_when_all_are_predicted():
    w = Window(3)
    for e in range(3):
        w.publish(e, e)
    assert w.plan([2, 3], {0}) == [(3, 1)]
    assert w.plan([2, 3], {0, 1}) == [(3, 0)]
    w.touch(0)
    assert w.plan([2, 3]) == [(3, 1)]
    with pytest.raises(StoreError):
        Window(2).plan([1, 2, 3])


def test_skipped_routes_do_not_displace_the_prompt_tail():
    assert tail_experts([1, 2, 3, 4, 5], [1.0, 1.0, 0.0, 0.0, 0.0], 2) == {1, 2}


def test_prompt_seed_uses_recent_unique_experts():
    assert tail_experts([0, 0, 0, 1, 2, 3, 2], [1.0] * 7, 3) == {1, 2, 3}
