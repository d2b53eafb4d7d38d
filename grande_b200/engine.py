"""The reference's Rust API (crates/omg-wgpu: ``EngineBuilder``, ``Engine``,
``SavedState``, ``QTensor``, ``Group``; crates/omg-core: ``BranchTokens``,
``Want``, ``PrefixSource``, ``Backend``) over the C ABI of
``include/omg_b200.h``. Same names, argument meanings and error messages;
errors raise :class:`OmgError` with the engine's message."""
from __future__ import annotations

import ctypes as C
import json
import threading
from itertools import chain
from dataclasses import dataclass, field
from enum import IntEnum
from typing import Optional, Sequence

import numpy as np

from . import _lib
from ._lib import OmgError, check, lib

SEQ_GROUP_SHIFT = 12  # engine.rs:21-24


class Dtype(IntEnum):
    """model.rs:338-371 (``Dtype::code``)."""
    F16 = 0
    Q8 = 1
    Q4 = 2

    @staticmethod
    def parse(s: str) -> "Dtype":
        m = {"f16": 0, "F16": 0, "q8": 1, "q8_0": 1, "Q8_0": 1, "q4": 2, "q4_0": 2, "Q4_0": 2}
        if s not in m:
            raise OmgError(f"unsupported dtype {s}")
        return Dtype(m[s])

    def payload_bytes(self, n: int) -> int:
        return n * 2 if self == Dtype.F16 else (n if self == Dtype.Q8 else n // 2)


class Want(IntEnum):
    """omg_core::Want (backend.rs:15-20)."""
    LOGITS = 0
    HIDDEN = 1


class PrefixSource(IntEnum):
    """omg_core::PrefixSource (backend.rs:95-104)."""
    RESIDENT = 0
    RAM = 1
    DISK = 2
    DECODED = 3

    def as_str(self) -> str:
        return self.name.lower()


def _source(v: int) -> Optional[PrefixSource]:
    return None if v < 0 else PrefixSource(v)


@dataclass
class BranchTokens:
    """omg_core::BranchTokens (backend.rs:26-30)."""
    tokens: Sequence[int]
    want: Sequence[int]


@dataclass
class BranchOutput:
    """omg_core::BranchOutput (backend.rs:34-36): rows in ``want`` order."""
    rows: np.ndarray


@dataclass
class Group:
    """omg_wgpu::Group (engine.rs:26-38)."""
    prefix: Sequence[int]
    branches: Sequence[BranchTokens]

    def tokens(self) -> int:
        return len(self.prefix) + sum(len(b.tokens) for b in self.branches)

    def rows(self) -> int:
        return sum(len(b.want) for b in self.branches)


@dataclass
class GroupOutput:
    """omg_core::GroupOutput (backend.rs:64-69)."""
    branches: list
    prefix_source: Optional[PrefixSource]


@dataclass
class QTensor:
    """model.rs:376-384: raw little-endian payload plus f16 block scales."""
    dtype: Dtype
    shape: list
    data: bytes
    scales: bytes = b""

    def numel(self) -> int:
        return int(np.prod(self.shape))

    @staticmethod
    def from_f32(shape, values) -> "QTensor":
        return QTensor._encode(Dtype.F16, shape, values)

    @staticmethod
    def quantize_q8(shape, values) -> "QTensor":
        return QTensor._encode(Dtype.Q8, shape, values)

    @staticmethod
    def quantize_q4(shape, values) -> "QTensor":
        return QTensor._encode(Dtype.Q4, shape, values)

    @staticmethod
    def _encode(dtype: Dtype, shape, values) -> "QTensor":
        v = np.ascontiguousarray(values, dtype=np.float32).ravel()
        n = v.size
        if dtype != Dtype.F16 and n % 32:
            raise OmgError(f"{dtype.name.lower()}: {n} values is not a multiple of 32")
        codes = np.empty(dtype.payload_bytes(n), dtype=np.uint8)
        scales = np.empty(0 if dtype == Dtype.F16 else n // 16, dtype=np.uint8)
        check(lib().omg_quantize(int(dtype), _lib.ptr(v, C.c_float), n,
                                 _lib.ptr(codes, C.c_uint8),
                                 _lib.ptr(scales, C.c_uint8) if scales.size else None))
        return QTensor(dtype, list(shape), codes.tobytes(), scales.tobytes())

    @staticmethod
    def from_raw(dtype: Dtype, shape, data: bytes, scales: bytes = b"") -> "QTensor":
        n = int(np.prod(shape))
        dtype = Dtype(dtype)
        if len(data) != dtype.payload_bytes(n):
            raise OmgError(f"{dtype!r} tensor {list(shape)}: {len(data)} payload bytes, "
                           f"expected {dtype.payload_bytes(n)}")
        want = 0 if dtype == Dtype.F16 else n // 32 * 2
        if len(scales) != want:
            raise OmgError(f"{dtype!r} tensor {list(shape)}: {len(scales)} scale bytes, "
                           f"expected {want}")
        return QTensor(dtype, list(shape), bytes(data), bytes(scales))

    def to_f32(self) -> np.ndarray:
        n = self.numel()
        out = np.empty(n, dtype=np.float32)
        d = np.frombuffer(self.data, dtype=np.uint8)
        s = np.frombuffer(self.scales, dtype=np.uint8) if self.scales else None
        check(lib().omg_dequantize(int(self.dtype), _lib.ptr(d, C.c_uint8),
                                   _lib.ptr(s, C.c_uint8) if s is not None else None, n,
                                   _lib.ptr(out, C.c_float)))
        return out

    def get(self, i: int) -> float:
        return float(self.to_f32()[i])


def _shape(shape) -> C.Array:
    return (C.c_int64 * len(shape))(*[int(s) for s in shape])


def _buf(b: bytes):
    return C.c_char_p(b) if b else None


class _HostBlock:
    """One page-locked block handed out as the base of an output array; it
    goes back to its pool when the last view of the array is gone."""

    __slots__ = ("pool", "addr", "size", "__array_interface__")

    def __init__(self, pool: "_HostPool", addr: int, size: int, shape):
        self.pool, self.addr, self.size = pool, addr, size
        self.__array_interface__ = {"shape": tuple(shape), "typestr": "<f4",
                                    "data": (addr, False), "version": 3}

    def __del__(self):
        try:
            self.pool.put(self.addr, self.size)
        except Exception:  # interpreter shutdown
            pass


class _HostPool:
    """Page-locked output arrays (omg_host_alloc on the engine's device),
    reused across calls: the engine copies the rows into them straight from
    the device. Blocks are sized in 64 KiB steps; a few free blocks per size
    are kept, the rest released."""

    STEP = 1 << 16
    KEEP = 4

    def __init__(self, device: int):
        self.device = device
        self.free: dict = {}
        # Re-entrant: a _HostBlock finalised by the cyclic collector while
        # this thread holds the lock (the collector may run on any
        # allocation) calls put() on the same thread.
        self.lock = threading.RLock()

    def array(self, shape) -> np.ndarray:
        size = max(int(np.prod(shape)) * 4, 1)
        size = (size + self.STEP - 1) // self.STEP * self.STEP
        with self.lock:
            blocks = self.free.get(size)
            addr = blocks.pop() if blocks else None
        if addr is None:
            ptr = C.c_void_p()
            if lib().omg_host_alloc(self.device, size, C.byref(ptr)) < 0:
                # Out of page-locked memory: a pageable array (staged copy).
                return np.empty(shape, dtype=np.float32)
            addr = ptr.value
        return np.asarray(_HostBlock(self, addr, size, shape))

    def put(self, addr: int, size: int):
        with self.lock:
            blocks = self.free.setdefault(size, [])
            if len(blocks) < self.KEEP:
                blocks.append(addr)
                return
        lib().omg_host_free(addr)


_POOLS: dict = {}
_POOLS_LOCK = threading.Lock()


def _host_pool(device: int) -> _HostPool:
    """The page-locked output pool of one device, shared by its engines."""
    with _POOLS_LOCK:
        if device not in _POOLS:
            _POOLS[device] = _HostPool(device)
        return _POOLS[device]


class _Branches:
    """Keeps the ctypes arrays of a request alive for one call."""

    def __init__(self, groups: Sequence[Group]):
        self.keep = []
        self.groups = (_lib.GroupC * len(groups))()
        for gi, g in enumerate(groups):
            prefix = np.fromiter(g.prefix, dtype=np.uint32, count=len(g.prefix))
            nb = len(g.branches)
            brs = (_lib.Branch * max(1, nb))()
            # One array for all branch tokens and one for all wanted rows; each
            # branch points at its slice.
            ntok = [len(b.tokens) for b in g.branches]
            nwant = [len(b.want) for b in g.branches]
            toks = np.fromiter(chain.from_iterable(b.tokens for b in g.branches),
                               dtype=np.int32, count=sum(ntok))
            wants = np.fromiter(chain.from_iterable(b.want for b in g.branches),
                                dtype=np.uint64, count=sum(nwant))
            tb, wb = toks.ctypes.data, wants.ctypes.data
            to = wo = 0
            for bi in range(nb):
                br = brs[bi]
                br.tokens = tb + 4 * to
                br.n_tokens = ntok[bi]
                br.want = wb + 8 * wo
                br.n_want = nwant[bi]
                to += ntok[bi]
                wo += nwant[bi]
            self.keep += [prefix, brs, toks, wants]
            self.groups[gi].prefix = _lib.ptr(prefix, C.c_uint32)
            self.groups[gi].n_prefix = prefix.size
            self.groups[gi].branches = brs
            self.groups[gi].n_branches = nb


class SavedState:
    """engine.rs:503-580 (a handle on the engine-side state)."""

    def __init__(self, handle):
        self._h = handle

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h:
            lib().omg_state_free(h)

    def byte_len(self) -> int:
        return int(lib().omg_state_byte_len(self._h))

    @property
    def prefix(self) -> list:
        n = C.c_size_t(0)
        check(lib().omg_state_prefix(self._h, None, 0, C.byref(n)))
        buf = np.empty(n.value, dtype=np.uint32)
        check(lib().omg_state_prefix(self._h, _lib.ptr(buf, C.c_uint32), n.value, C.byref(n)))
        return buf.tolist()

    def to_bytes(self, model_id: str) -> bytes:
        need = C.c_size_t(0)
        mid = model_id.encode()
        check(lib().omg_state_to_bytes(self._h, mid, None, 0, C.byref(need)))
        buf = (C.c_uint8 * need.value)()
        check(lib().omg_state_to_bytes(self._h, mid, buf, need.value, C.byref(need)))
        return bytes(buf)

    @staticmethod
    def from_bytes(data: bytes, model_id: str) -> "SavedState":
        h = C.c_void_p()
        arr = (C.c_uint8 * len(data)).from_buffer_copy(data)
        check(lib().omg_state_from_bytes(arr, len(data), model_id.encode(), C.byref(h)))
        return SavedState(h)


class Engine:
    """engine.rs:449-2171 on one B200."""

    def __init__(self, handle):
        self._h = handle
        info = _lib.EngineInfo()
        check(lib().omg_engine_get_info(self._h, C.byref(info)))
        self.d = info.d
        self.vocab = info.vocab
        self.layers = info.layers
        self.capacity = info.capacity
        self.max_rows = info.max_rows
        self.per_layer_dim = info.per_layer_dim
        self.device = info.device
        self.bos = info.bos
        self._embed_dtype = Dtype(info.embed_dtype)
        self._pool = _host_pool(self.device)

    def close(self):
        h, self._h = getattr(self, "_h", None), None
        if h:
            lib().omg_engine_destroy(h)

    def __del__(self):
        self.close()

    @staticmethod
    def new(weights: "dict[str, QTensor]", config_json: str, capacity: int, max_rows: int,
            device: int = 0, per_layer_table: Optional[QTensor] = None) -> "Engine":
        """Engine::new (engine.rs:1338-1349): upload a whole host checkpoint."""
        b = EngineBuilder(config_json, device)
        for name in b.catalogue():
            if name not in weights:
                raise OmgError(f"missing tensor {name}")
            b.push(name, weights[name])
        if per_layer_table is not None:
            b.set_per_layer_table(per_layer_table)
        return b.finish(capacity, max_rows)

    def embed_dtype(self) -> Dtype:
        return self._embed_dtype

    def _run(self, groups: Sequence[Group], want: Want, rows: Optional[bytes] = None):
        req = _Branches(groups)
        width = self.vocab if Want(want) == Want.LOGITS else self.d
        nrows = sum(g.rows() for g in groups)
        out = self._pool.array((max(nrows, 1), width))
        srcs = (C.c_int32 * len(groups))()
        if rows is None:
            check(lib().omg_engine_evaluate_groups(self._h, req.groups, len(groups), int(want),
                                                   _lib.ptr(out, C.c_float), out.size, srcs))
        else:
            g = req.groups[0]
            arr = (C.c_uint8 * len(rows)).from_buffer_copy(rows) if rows else None
            check(lib().omg_engine_evaluate_rows(self._h, g.prefix, g.n_prefix, g.branches,
                                                 g.n_branches, int(want), arr, len(rows),
                                                 _lib.ptr(out, C.c_float), out.size))
        outs, r = [], 0
        for gi, grp in enumerate(groups):
            brs = []
            for b in grp.branches:
                # Views into this call's own output array (no second copy).
                brs.append(BranchOutput(out[r:r + len(b.want)]))
                r += len(b.want)
            outs.append(GroupOutput(brs, _source(srcs[gi]) if rows is None else None))
        return outs

    def evaluate(self, prefix, branches, want: Want) -> list:
        """engine.rs:1386-1398."""
        return self._run([Group(prefix, branches)], want)[0].branches

    def evaluate_groups(self, groups: Sequence[Group], want: Want) -> list:
        """engine.rs:1404-1444."""
        if not groups:
            raise OmgError("empty request")
        return self._run(groups, want)

    def evaluate_rows(self, prefix, branches, want: Want, per_layer_rows: Optional[bytes]):
        """engine.rs:1449-1463."""
        return self._run([Group(prefix, branches)], want, per_layer_rows or b"")[0].branches

    def warmup(self):
        check(lib().omg_engine_warmup(self._h))

    def prefix_source(self) -> Optional[PrefixSource]:
        return _source(lib().omg_engine_prefix_source(self._h))

    def is_resident(self, prefix) -> bool:
        p = np.ascontiguousarray(np.asarray(prefix, dtype=np.int64).astype(np.uint32))
        return bool(lib().omg_engine_is_resident(self._h, _lib.ptr(p, C.c_uint32), p.size))

    def evict_resident(self):
        lib().omg_engine_evict_resident(self._h)

    def set_state_cache(self, nbytes: int, dir: Optional[str], model_id: str):
        check(lib().omg_engine_set_state_cache(self._h, nbytes, (dir or "").encode(),
                                               model_id.encode()))

    def save_state(self, prefix) -> SavedState:
        p = np.ascontiguousarray(np.asarray(prefix, dtype=np.int64).astype(np.uint32))
        h = C.c_void_p()
        check(lib().omg_engine_save_state(self._h, _lib.ptr(p, C.c_uint32), p.size, C.byref(h)))
        return SavedState(h)

    def restore_state(self, state: SavedState):
        check(lib().omg_engine_restore_state(self._h, state._h))

    # ---- a state moved between GPUs (no host copy) ----------------------------

    def state_image_bytes(self, n_prefix: int) -> int:
        """Bytes of the device image of an `n_prefix`-token state (the f16 K/V
        rows save_state returns, layer payloads concatenated)."""
        return int(lib().omg_engine_state_image_bytes(self._h, n_prefix))

    def export_state_device(self, prefix, dst_ptr: int, cap: int):
        """Copy the resident `prefix`'s K/V rows into device memory at
        `dst_ptr` (this engine's GPU); complete on return."""
        p = np.ascontiguousarray(np.asarray(prefix, dtype=np.int64).astype(np.uint32))
        check(lib().omg_engine_export_state_device(self._h, _lib.ptr(p, C.c_uint32), p.size,
                                                   C.c_void_p(dst_ptr), cap))

    def import_state_device(self, prefix, src_ptr: int, nbytes: int):
        """Make `prefix` resident from a device image at `src_ptr` (this
        engine's GPU), as restore_state does from a SavedState."""
        p = np.ascontiguousarray(np.asarray(prefix, dtype=np.int64).astype(np.uint32))
        check(lib().omg_engine_import_state_device(self._h, _lib.ptr(p, C.c_uint32), p.size,
                                                   C.c_void_p(src_ptr), nbytes))

    def gather_per_layer(self, ids) -> bytes:
        i = np.ascontiguousarray(np.asarray(ids, dtype=np.int64).astype(np.uint32))
        n = i.size * self.per_layer_dim * self.layers * 2
        out = np.empty(n, dtype=np.uint8)
        check(lib().omg_engine_gather_per_layer(self._h, _lib.ptr(i, C.c_uint32), i.size,
                                                _lib.ptr(out, C.c_uint8), n))
        return out.tobytes()

    def arm_wait_timeout(self, clocks: int):
        """Test hook: the next pass's first fused FFN launch waits for a band
        that never completes and gives up after `clocks` SM clocks, so that
        pass raises the engine's wait-timeout error."""
        check(lib().omg_engine_arm_wait_timeout(self._h, int(clocks)))

    def weight_f16(self, name: str, shape) -> np.ndarray:
        """The f16 bits the projection GEMMs multiply for linear `name`
        ([rows, k] uint16), read back from the device."""
        out = np.empty(tuple(shape), dtype=np.uint16)
        check(lib().omg_engine_weight_f16(self._h, name.encode(), _lib.ptr(out, C.c_uint16),
                                          out.size))
        return out

    # ---- timing hooks (bench.py) --------------------------------------------

    def time_forward(self, groups: Sequence[Group], want: Want, iters: int,
                     resident: bool = False) -> tuple[float, int]:
        req = _Branches(groups)
        ms = C.c_float(0)
        launches = C.c_int(0)
        check(lib().omg_engine_time_forward(self._h, req.groups, len(groups), int(want),
                                            int(resident), iters, C.byref(ms),
                                            C.byref(launches)))
        return ms.value, launches.value

    def profile_forward(self, groups: Sequence[Group], want: Want, iters: int,
                        resident: bool = False) -> dict:
        """Per-kernel device time: {name: (launches, total_ms)}."""
        req = _Branches(groups)
        need = C.c_size_t(0)
        buf = C.create_string_buffer(8192)
        check(lib().omg_engine_profile_forward(self._h, req.groups, len(groups), int(want),
                                               int(resident), iters, buf, 8192, C.byref(need)))
        return {k: tuple(v) for k, v in json.loads(buf.value.decode()).items()}

    def record_event(self, slot: int):
        check(lib().omg_engine_record_event(self._h, slot))

    def elapsed_ms(self, a: int, b: int) -> float:
        ms = C.c_float(0)
        check(lib().omg_engine_elapsed_ms(self._h, a, b, C.byref(ms)))
        return ms.value


class EngineBuilder:
    """engine.rs:805-1334."""

    def __init__(self, config_json: str, device: int = 0):
        if isinstance(config_json, dict):
            config_json = json.dumps(config_json)
        self.config_json = config_json
        h = C.c_void_p()
        check(lib().omg_builder_new(config_json.encode(), device, C.byref(h)))
        self._h = h

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h:
            lib().omg_builder_free(h)

    def catalogue(self) -> list:
        return [n for n, _ in config_tensors(self.config_json)]

    def set_weight_layout(self, packed: bool):
        """Q4_0 / Q8_0 linears pushed from now on: kept packed and decoded
        per tile in shared memory by the GEMMs (True; 18 bytes per 32 Q4_0
        weights), or decoded once into f16 rows (False, the default: faster,
        3.6x the memory). Same results either way."""
        check(lib().omg_builder_set_weight_layout(self._h, 0 if packed else 1))

    def push(self, name: str, t: QTensor):
        shape = _shape(t.shape)
        check(lib().omg_builder_push(self._h, name.encode(), int(t.dtype), shape, len(t.shape),
                                     _buf(t.data), len(t.data), _buf(t.scales), len(t.scales)))

    def set_per_layer_table(self, t: QTensor):
        shape = _shape(t.shape)
        check(lib().omg_builder_set_per_layer_table(self._h, int(t.dtype), shape, len(t.shape),
                                                    _buf(t.data), len(t.data), _buf(t.scales),
                                                    len(t.scales)))

    def missing(self) -> list:
        need = C.c_size_t(0)
        check(lib().omg_builder_missing(self._h, None, 0, C.byref(need)))
        buf = C.create_string_buffer(need.value)
        check(lib().omg_builder_missing(self._h, buf, need.value, C.byref(need)))
        return [s for s in buf.value.decode().split("\n") if s]

    def finish(self, capacity: int, max_rows: int) -> Engine:
        h = C.c_void_p()
        b, self._h = self._h, None
        check(lib().omg_builder_finish(b, capacity, max_rows, C.byref(h)))
        return Engine(h)


def config_tensors(config_json: str) -> list:
    """Config::tensors (model.rs:277-314): [(name, shape)]."""
    need = C.c_size_t(0)
    check(lib().omg_config_tensors(config_json.encode(), None, 0, C.byref(need)))
    buf = C.create_string_buffer(need.value)
    check(lib().omg_config_tensors(config_json.encode(), buf, need.value, C.byref(need)))
    out = []
    for line in buf.value.decode().split("\n"):
        if line:
            name, dims = line.split(" ")
            out.append((name, [int(x) for x in dims.split(",")]))
    return out


def state_key(model_id: str, prefix) -> int:
    p = np.ascontiguousarray(np.asarray(prefix, dtype=np.int64).astype(np.uint32))
    return int(lib().omg_state_key(model_id.encode(), _lib.ptr(p, C.c_uint32), p.size))


@dataclass
class Limits:
    """omg_core::Limits (backend.rs:73-80)."""
    tokens: int
    sequences: int
    rows: int


class B200Backend:
    """omg_core::Backend (backend.rs:117-167) over the engine, as
    WgpuBackend (crates/omg-wgpu/src/backend.rs:203-285) is over wgpu.
    Tokenization is the caller's (token ids in, rows out)."""

    def __init__(self, engine: Engine):
        self.engine = engine

    def bos(self) -> int:
        return self.engine.bos

    def n_embd(self) -> int:
        return self.engine.d

    def n_vocab(self) -> int:
        return self.engine.vocab

    def evaluate(self, prefix, branches, want: Want) -> list:
        return self.engine.evaluate(prefix, branches, want)

    def evaluate_many(self, groups: Sequence[Group], want: Want) -> list:
        return self.engine.evaluate_groups(groups, want)

    def limits(self) -> Limits:
        return Limits(self.engine.capacity, 2**63 - 1, self.engine.max_rows)

    def prefix_source(self) -> Optional[PrefixSource]:
        return self.engine.prefix_source()

    def evict_resident(self):
        self.engine.evict_resident()

    @staticmethod
    def load(dir, capacity: int, max_rows: int, device: int = 0) -> "B200Backend":
        """WgpuBackend::load (crates/omg-wgpu/src/backend.rs:25-63) without
        the tokenizer: an exported directory or a Gemma 3 safetensors
        checkpoint, warmed up."""
        from .checkpoint import load_engine
        return B200Backend(load_engine(dir, capacity, max_rows, device))

    def set_state_cache(self, dir_path, nbytes: int, dir: Optional[str] = None):
        """backend.rs:80-96: the model id is the checkpoint directory's name
        and the byte size of its tensor files."""
        from .checkpoint import model_id
        self.engine.set_state_cache(nbytes, dir, model_id(dir_path))
