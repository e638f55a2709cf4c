"""Expert paging: the on-disk record store, the per-layer slot window and a
pager that runs a layer whose experts do not all fit in one slot bank.

Restates (happyme531/open_rknpu2_lm_infer):
  Store / Writer / Record / lock : src/model/experts/store.rs (the experts.npu
      container: magic, JSON header, page-aligned positional records)
  Window / tail_experts          : src/model/experts/window.rs (LRU slots; the
      requested experts are pinned; eviction avoids predicted experts first)
  Pager                          : src/model/experts/paged.rs:234-540 (demand,
      plan, import into slots, per-assignment expert rows, one reduction in
      rank order)

The records are this library's expert blobs (moe_b200_export_expert), so a
store is tied to MOE_B200_BLOB_VERSION through Geometry.native_version. The
pager computes every assignment's expert row with the expert-parallel entry
points (pack, expert rows over slot ids, combine), so its output equals the
resident layer bit for bit whatever the slot count.
"""
from __future__ import annotations

import fcntl
import json
import mmap
import os
import struct
from dataclasses import asdict, dataclass
from pathlib import Path

import numpy as np

PAGE = 4096
MAGIC = b"RKMOE01\0"
FILE = "experts.npu"


class StoreError(ValueError):
    pass


def _ensure(cond, msg):
    if not cond:
        raise StoreError(msg)


@dataclass
class Geometry:
    native_version: int
    layers: int
    experts: int
    hidden: int
    intermediate: int
    down_bits: int = 4
    packing_revision: int = 0

    def to_json(self) -> dict:
        d = asdict(self)
        if d["packing_revision"] == 0:
            del d["packing_revision"]  # skipped when zero (store.rs:21-24)
        return d

    @staticmethod
    def from_json(d: dict) -> "Geometry":
        return Geometry(d["native_version"], d["layers"], d["experts"], d["hidden"],
                        d["intermediate"], d["down_bits"], d.get("packing_revision", 0))


def lock(directory) -> object:
    """Exclusive lock of a cache directory while it is built (store.rs:319-333)."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    fh = open(directory / "prepare.lock", "a+b")
    fcntl.flock(fh.fileno(), fcntl.LOCK_EX)
    return fh


class Writer:
    """Writes records in (layer, expert) order, then publishes the file by
    rename (store.rs:335-431)."""

    def __init__(self, directory, geometry: Geometry, sources, record_bytes: int):
        _ensure(record_bytes > 0, "empty expert record")
        directory = Path(directory)
        directory.mkdir(parents=True, exist_ok=True)
        stride = -(-record_bytes // PAGE) * PAGE
        header = {"geometry": geometry.to_json(), "sources": [list(s) for s in sources],
                  "record_bytes": record_bytes, "record_stride": stride, "data_offset": PAGE}
        while True:
            blob = json.dumps(header, separators=(",", ":")).encode()
            offset = -(-(16 + len(blob)) // PAGE) * PAGE
            if header["data_offset"] == offset:
                break
            header["data_offset"] = offset
        self.header = header
        self.geometry = geometry
        self.path = directory / f"{FILE}.tmp.{os.getpid()}"
        self.final_path = directory / FILE
        self.fh = open(self.path, "wb")
        self.fh.write(MAGIC)
        self.fh.write(struct.pack("<Q", len(blob)))
        self.fh.write(blob)
        self.fh.write(b"\0" * (offset - 16 - len(blob)))
        self.written = 0
        self.finished = False

    def write(self, layer: int, expert: int, data) -> None:
        g = self.geometry
        data = bytes(data)
        _ensure(self.written == layer * g.experts + expert and layer < g.layers and
                expert < g.experts and len(data) == self.header["record_bytes"],
                "expert export order/size mismatch")
        self.fh.write(data)
        self.fh.write(b"\0" * (self.header["record_stride"] - len(data)))
        self.written += 1

    def finish(self) -> None:
        g = self.geometry
        _ensure(self.written == g.layers * g.experts, "missing exported experts")
        self.fh.flush()
        os.fsync(self.fh.fileno())
        self.fh.close()
        os.replace(self.path, self.final_path)
        self.finished = True

    def __del__(self):
        if not getattr(self, "finished", True):
            try:
                self.fh.close()
                os.unlink(self.path)
            except OSError:
                pass


class Record:
    """A page-aligned read buffer holding one record; returned to its store's
    pool on release (store.rs:268-293)."""

    def __init__(self, buf: mmap.mmap, raw: int, pool: "Store"):
        self._buf = buf
        self.raw = raw
        self._pool = pool

    def as_bytes(self) -> memoryview:
        return memoryview(self._buf)[: self.raw]

    def address(self) -> int:
        import ctypes
        return ctypes.addressof(ctypes.c_char.from_buffer(self._buf))

    def release(self) -> None:
        if self._buf is not None:
            self._pool._give_back(self._buf)
            self._buf = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.release()

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class Store:
    """Reads positional expert records (store.rs:44-230)."""

    def __init__(self, directory, geometry: Geometry, sources, direct: bool = False):
        path = Path(directory) / FILE
        self.fd = os.open(path, os.O_RDONLY | (os.O_DIRECT if direct else 0))
        try:
            self._open(geometry, sources, direct)
        except Exception:
            self.close()
            raise

    def _open(self, geometry: Geometry, sources, direct: bool) -> None:
        size = os.fstat(self.fd).st_size
        prefix = os.pread(self.fd, 16, 0) if not direct else self._aligned_read(0, PAGE)[:16]
        _ensure(len(prefix) == 16 and prefix[:8] == MAGIC, "not a native expert cache")
        (length,) = struct.unpack("<Q", prefix[8:])
        _ensure(length <= max(size - 16, 0), "truncated expert header")
        raw = (os.pread(self.fd, length, 16) if not direct
               else self._aligned_read(0, -(-(16 + length) // PAGE) * PAGE)[16:16 + length])
        header = json.loads(raw)
        hg = Geometry.from_json(header["geometry"])
        _ensure(hg.native_version == geometry.native_version,
                f"expert cache format v{hg.native_version} requires rebuilding for "
                f"v{geometry.native_version}")
        _ensure(hg.packing_revision == geometry.packing_revision,
                f"expert cache packing revision {hg.packing_revision} requires rebuilding for "
                f"{geometry.packing_revision}")
        _ensure(hg == geometry and [tuple(s) for s in header["sources"]] ==
                [tuple(s) for s in sources] and geometry.down_bits in (4, 8),
                "expert cache does not match checkpoint/recipe")
        rb, rs, off = header["record_bytes"], header["record_stride"], header["data_offset"]
        _ensure(0 < rb <= rs and rs % PAGE == 0 and off % PAGE == 0 and off >= 16 + length,
                "invalid expert record layout")
        _ensure(size == off + geometry.layers * geometry.experts * rs, "incomplete expert cache")
        self.geometry = geometry
        self.record_bytes, self.record_stride, self.data_offset = rb, rs, off
        self._free: list[mmap.mmap] = []
        self.allocations = 0
        self.reuses = 0

    def _aligned_read(self, offset: int, length: int) -> bytes:
        buf = mmap.mmap(-1, length)
        os.preadv(self.fd, [buf], offset)
        return bytes(buf)

    def close(self) -> None:
        if self.fd >= 0:
            os.close(self.fd)
            self.fd = -1

    def _buffer(self) -> mmap.mmap:
        if self._free:
            self.reuses += 1
            return self._free.pop()
        self.allocations += 1
        return mmap.mmap(-1, self.record_stride)  # page-aligned anonymous memory

    def _give_back(self, buf) -> None:
        if len(self._free) < 32:
            self._free.append(buf)

    def buffer_stats(self) -> dict:
        return {"allocations": self.allocations, "reuses": self.reuses,
                "idle_buffers": len(self._free),
                "idle_bytes": len(self._free) * self.record_stride}

    def _offset(self, layer: int, expert: int) -> int:
        return self.data_offset + (layer * self.geometry.experts + expert) * self.record_stride

    def read(self, layer: int, expert: int) -> Record:
        g = self.geometry
        _ensure(0 <= layer < g.layers and 0 <= expert < g.experts, "expert file index out of range")
        buf = self._buffer()
        got = os.preadv(self.fd, [buf], self._offset(layer, expert))
        _ensure(got == self.record_stride, f"read expert {layer}/{expert}")
        return Record(buf, self.record_bytes, self)

    def read_batch(self, layer: int, first: int, count: int) -> list[Record]:
        """Neighbouring records with one vectored read (store.rs:166-213)."""
        g = self.geometry
        _ensure(count > 0 and 0 <= layer < g.layers and 0 <= first and first + count <= g.experts,
                "expert batch out of range")
        bufs = [self._buffer() for _ in range(count)]
        total, done = count * self.record_stride, 0
        off = self._offset(layer, first)
        while done < total:
            views, skip = [], done
            for b in bufs:
                if skip >= len(b):
                    skip -= len(b)
                    continue
                views.append(memoryview(b)[skip:])
                skip = 0
            got = os.preadv(self.fd, views, off + done)
            _ensure(got > 0, "truncated expert batch")
            done += got
        return [Record(b, self.record_bytes, self) for b in bufs]


class Window:
    """Per-layer LRU slot window (window.rs:9-100): requested experts are
    pinned, empty slots are used first, then the least recently used slot
    whose expert is neither requested nor (if possible) predicted."""

    def __init__(self, slots: int):
        self.contents: list[int | None] = [None] * slots
        self.age = [0] * slots
        self.clock = 0

    def slot(self, expert: int) -> int | None:
        try:
            return self.contents.index(expert)
        except ValueError:
            return None

    def touch(self, expert: int) -> None:
        s = self.slot(expert)
        if s is not None:
            self.clock += 1
            self.age[s] = self.clock

    def publish(self, slot: int, expert: int) -> None:
        self.contents[slot] = expert
        self.touch(expert)

    def invalidate(self, slot: int) -> None:
        self.contents[slot] = None
        self.age[slot] = 0

    def victim(self, requested: set, predicted: set, reserved: set) -> int:
        for s, e in enumerate(self.contents):
            if e is None and s not in reserved:
                return s
        for protect in (True, False):
            cands = [s for s, e in enumerate(self.contents)
                     if s not in reserved and e is not None and e not in requested and
                     (not protect or e not in predicted)]
            if cands:
                return min(cands, key=lambda s: self.age[s])
        raise StoreError("expert window cannot hold this token's requested experts")

    def plan(self, requested: list[int], predicted: set = frozenset()) -> list[tuple[int, int]]:
        """(expert, slot) for every requested expert not resident."""
        req = set(requested)
        _ensure(len(req) <= len(self.contents), "expert window must hold at least one token's top-k")
        reserved, missing = set(), []
        for e in requested:
            if self.slot(e) is None:
                s = self.victim(req, set(predicted), reserved)
                reserved.add(s)
                missing.append((e, s))
        return missing


def tail_experts(ids, weights, capacity: int) -> set:
    """The last `capacity` distinct routed experts of a prompt (window.rs:103-117)."""
    out = set()
    for e, w in zip(reversed(list(ids)), reversed(list(weights))):
        if w == 0:
            continue
        out.add(int(e))
        if len(out) == capacity:
            break
    return out


@dataclass
class _LayerShape:
    """What the EP device steps read of a router: the layer's shape."""
    hidden: int
    experts: int
    top: int
    raw: object = None


@dataclass
class PagerStats:
    calls: int = 0
    assignments: int = 0
    hot_assignments: int = 0
    unique_demand: int = 0
    cold_experts: int = 0
    imports: int = 0
    groups: int = 0


class Pager:
    """One layer's routed experts paged through a bank of `slots` slots.

    run(x, ids, routes[, residual]) = the resident layer's output, bit for
    bit: the rows are quantised and packed once (moe_b200_ep_pack), every
    group of at most `slots` demanded experts is imported into the window's
    planned slots and its rows run through moe_b200_ep_expert_rows with slot
    ids, and one combine reduces each token's expert rows in rank order."""

    def __init__(self, backend, store: Store, layer: int, slots: int, top: int, fmt: int,
                 max_rows: int):
        import torch

        from .ep import DeviceOps
        g = store.geometry
        # the window holds at least one token's top-k (window.rs:85-88)
        _ensure(0 < top <= slots <= g.experts, "invalid hot expert slot count")
        self.torch = torch
        self.store, self.layer, self.top = store, layer, top
        self.hot = backend.moe_packed(g.hidden, g.intermediate, slots, top, fmt)
        self.window = Window(slots)
        self.experts = g.experts
        shape = _LayerShape(g.hidden, g.experts, top)
        self.ops = DeviceOps(backend, self.hot, shape, 1, max_rows)
        self.y_all = torch.empty((max_rows * top, g.hidden), dtype=torch.float32,
                                 device=self.ops.y.device)
        self.stats = PagerStats()

    def _import(self, expert: int, slot: int) -> None:
        with self.store.read(self.layer, expert) as rec:
            self.hot.import_(slot, rec.as_bytes())
        self.window.publish(slot, expert)
        self.stats.imports += 1

    def run(self, x, ids, routes, residual=None, predicted: set = frozenset()):
        """x [T][H] f32, ids [T][k] i32, routes [T][k] f32 (device tensors)."""
        torch = self.torch
        T = x.shape[0]
        ids_h = ids.cpu().numpy().reshape(-1)
        w_h = routes.cpu().numpy().reshape(-1)
        _ensure(((ids_h >= 0) & (ids_h < self.experts)).all(), "paged expert id out of range")
        kept = w_h > 0
        demand = list(dict.fromkeys(int(e) for e in ids_h[kept]))
        st = self.stats
        st.calls += 1
        st.assignments += int(kept.sum())
        st.hot_assignments += int(sum(1 for e in ids_h[kept] if self.window.slot(int(e)) is not None))
        st.unique_demand += len(demand)
        cold = [e for e in demand if self.window.slot(e) is None]
        st.cold_experts += len(cold)
        send_q, send_s, send_e, counts, pos = self.ops.pack(x, ids, routes)
        n = int(kept.sum())
        expert_rows = send_e[:n].cpu().numpy()  # world 1: the global expert id
        cap = len(self.window.contents)
        groups = [demand] if len(demand) <= cap else \
            [demand[i:i + cap] for i in range(0, len(demand), cap)]
        for group in groups:
            for expert, slot in self.window.plan(group, predicted):
                self.window.invalidate(slot)
                self._import(expert, slot)
            slot_of = np.full(self.experts, -1, np.int32)
            for e in group:
                slot_of[e] = self.window.slot(e)
            if len(groups) == 1:
                slots_dev = torch.from_numpy(slot_of[expert_rows]).to(x.device)
                y = self.ops.expert_rows(send_q[:n], send_s[:n], slots_dev)
            else:
                # this group's rows, then their expert rows scattered back in place
                sel = np.flatnonzero(np.isin(expert_rows, group))
                rows = torch.from_numpy(sel.astype(np.int64)).to(x.device)
                slots_dev = torch.from_numpy(slot_of[expert_rows[sel]]).to(x.device)
                yg = self.ops.expert_rows(send_q[rows].contiguous(), send_s[rows].contiguous(),
                                          slots_dev)
                self.y_all[rows] = yg
                y = self.y_all[:n]
            st.groups += 1
        for e in ids_h[kept]:
            self.window.touch(int(e))
        return self.ops.combine(y, pos, routes, residual)

    def close(self):
        self.ops.close()
        self.hot.close()
