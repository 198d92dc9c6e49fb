"""ctypes binding of libgsp_b200.so, the C ABI declared in include/gsp_b200.h.

This is the only route from Python to the device: there is no Triton, no
PyTorch compute fallback and no CPU path. If the library is missing, or a
tensor is not on a CUDA device, calls raise instead of computing elsewhere.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libgsp_b200.so")

GSP_OK = 0
GSP_ERR_INVALID_ARGUMENT = -1
GSP_ERR_UNSUPPORTED = -2
GSP_ERR_WORKSPACE = -3
GSP_ERR_CUDA = -4
TILE_ROWS = 128

DTYPE_CODES = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}


class GSPNativeError(RuntimeError):
    """A C-ABI call returned an error status."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


_lib = None
_lib_lock = threading.Lock()

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t

class RouteCost(ctypes.Structure):
    """gsp_route_cost: the device route selector's cost model (us, GB/s)."""
    _fields_ = [(name, ctypes.c_double) for name in (
        "hbm_gbs", "row_sparse_fixed_us", "block_floor_us", "block_fixed_us", "block_gbs",
        "dense_fixed_us", "dense_gbs", "group_split_fixed_us")]


_PROJECTION_ARGS = [_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _i64,
                    _vp, _i64, _vp, _vp, _vp, _vp, _sz, _vp]

SIGNATURES = {
    "gsp_abi_version": ([], _i32),
    "gsp_status_string": ([_i32], ctypes.c_char_p),
    "gsp_last_error": ([], ctypes.c_char_p),
    "gsp_workspace_bytes": ([_i32, _i32], _sz),
    "gsp_row_sparse_logits": (_PROJECTION_ARGS, _i32),
    "gsp_row_sparse_compact": ([_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _i64,
                                _vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _sz, _vp], _i32),
    "gsp_ids_to_bitmask": ([_vp, _i64, _i32, _vp, _vp, _vp], _i32),
    "gsp_mask_stats": ([_vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp], _i32),
    "gsp_block_gemm_logits": (_PROJECTION_ARGS, _i32),
    "gsp_dense_masked_logits": (_PROJECTION_ARGS, _i32),
    "gsp_top1_from_keys": ([_vp, _i32, _vp, _vp, _vp], _i32),
    "gsp_row_sparse_logits_static": ([_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _i64,
                                      _vp, _i64, _vp, _vp, _vp, _vp], _i32),
    "gsp_row_sparse_static_error": ([ctypes.POINTER(_i32), _vp], _i32),
    "gsp_row_sparse_sample": ([_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _i64, _vp, _i64,
                               ctypes.c_float, _vp, ctypes.c_uint64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz,
                               _vp], _i32),
    "gsp_merge_logsumexp": ([_vp, _i32, _i32, _vp, _vp], _i32),
    "gsp_sample": ([_i32, _vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _i64, _vp, _i64,
                    ctypes.c_float, _vp, ctypes.c_uint64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp], _i32),
    "gsp_peer_exchange_bytes": ([_i32, _i32], _sz),
    "gsp_peer_exchange_alloc": ([_sz, ctypes.POINTER(_vp), _vp], _i32),
    "gsp_peer_exchange_open": ([_vp, ctypes.POINTER(_vp)], _i32),
    "gsp_peer_exchange_close": ([_vp], _i32),
    "gsp_peer_exchange_free": ([_vp], _i32),
    "gsp_peer_exchange_reset": ([_vp, _i32, _i32], _i32),
    "gsp_vocab_parallel_logits": ([_i32] + _PROJECTION_ARGS[:-1] + [ctypes.POINTER(_vp), _i32, _i32, _i32, _i64,
                                                               _i64, _vp], _i32),
    "gsp_default_route_cost": ([ctypes.POINTER(RouteCost)], None),
    "gsp_choose_route": ([_i32, _i32, _i32, _i32, _i64, _i64, ctypes.POINTER(RouteCost)], _i32),
    "gsp_adaptive_logits": ([_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _vp, _i64, _vp, _vp,
                             ctypes.POINTER(RouteCost), _vp, ctypes.POINTER(_i32), _vp, _sz, _vp], _i32),
    "gsp_group_plan_words": ([_i32], _sz),
    "gsp_group_plan": ([_vp, _i64, _i32, _i32, _i32, _i32, _i32, ctypes.POINTER(RouteCost), _vp, _vp], _i32),
    "gsp_gather_rows": ([_vp, _i64, _vp, _i32, _i64, _vp, _i64, _vp], _i32),
    "gsp_copy_bytes": ([_vp, _vp, _sz, _vp], _i32),
    "gsp_row_sparse_step": ([_vp, _sz, _vp] + _PROJECTION_ARGS, _i32),
    "gsp_step_graph_create": ([ctypes.POINTER(_vp), _vp, _sz, _vp] + _PROJECTION_ARGS[:-1], _i32),
    "gsp_step_graph_launch": ([_vp, _vp, _vp], _i32),
    "gsp_step_graph_destroy": ([_vp], _i32),
    "gsp_grouped_scratch_bytes": ([_i32, _i32, _i32, _i32], _sz),
    "gsp_grouped_logits": ([_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _vp, _i64, _vp, _vp,
                            ctypes.POINTER(RouteCost), ctypes.POINTER(_i32), _vp, _sz, _vp, _sz, _vp], _i32),
}

ROUTE_CODES = {"row-sparse": 0, "block-sparse": 1, "dense-mask": 2}
IPC_HANDLE_BYTES = 64
MAX_PEERS = 8


def load() -> ctypes.CDLL:
    """Load the library once; raise loudly if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"libgsp_b200.so is not built (expected at {LIB_PATH}); run "
                    "`python grammar-sparse-projection_b200/build.py` or __graft_entry__.build()")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (args, res) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = res
            _lib = lib
    return _lib


def _check(status: int, fn: str) -> None:
    if status != GSP_OK:
        lib = load()
        msg = lib.gsp_last_error().decode(errors="replace")
        name = lib.gsp_status_string(status).decode()
        raise GSPNativeError(status, f"{fn} failed with {name}: {msg}")


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}: the B200 kernels take float16, bfloat16 or float32") from None


# ---------------------------------------------------------------------------
# workspace: one zero-initialised buffer per (device, stream); every kernel
# leaves it zeroed again, so stream order makes reuse safe.
# ---------------------------------------------------------------------------
_workspaces: dict[tuple[int, int], torch.Tensor] = {}
_ws_lock = threading.Lock()


def workspace(device: torch.device, batch: int, vocab: int) -> torch.Tensor:
    need = int(load().gsp_workspace_bytes(batch, vocab))
    dev_index = device.index if device.index is not None else torch.cuda.current_device()
    key = (dev_index, torch.cuda.current_stream(device).cuda_stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < need:
            size = max(need, 64 * 1024, 0 if ws is None else 2 * ws.numel())
            ws = torch.zeros(size, dtype=torch.uint8, device=device)
            _workspaces[key] = ws
        return ws


def reset_workspace(device: torch.device) -> None:
    """Re-zeroes the current stream's workspace (needed after a call whose
    kernel reported an error through workspace_error)."""
    dev_index = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get((dev_index, torch.cuda.current_stream(device).cuda_stream))
    if ws is not None:
        ws.zero_()


def workspace_error(device: torch.device) -> int:
    """Error word of the current stream's workspace: non-zero after a kernel
    gave up a bounded wait (reads the device, so it synchronises)."""
    dev_index = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get((dev_index, torch.cuda.current_stream(device).cuda_stream))
    if ws is None:
        return 0
    return int(ws[4:8].view(torch.int32).item())


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and t.device.type != "cuda":
            raise ValueError("GSP B200 kernels take CUDA tensors only (no CPU path)")


# ---------------------------------------------------------------------------
# thin wrappers over the entry points (no validation beyond what the C ABI does)
# ---------------------------------------------------------------------------
def _projection(entry: str, hidden: torch.Tensor, weight: torch.Tensor, mask: torch.Tensor | None,
                logits: torch.Tensor | None, top_value: torch.Tensor | None,
                top_index: torch.Tensor | None, top_key: torch.Tensor | None,
                vocab_offset: int = 0) -> None:
    _require_cuda(hidden, weight, mask, logits)
    lib = load()
    batch, hdim = hidden.shape
    vocab = weight.shape[0]
    ws = workspace(hidden.device, batch, vocab)
    status = getattr(lib, entry)(
        _ptr(hidden), hidden.stride(0), _ptr(weight), weight.stride(0),
        _ptr(mask), 0 if mask is None else mask.stride(0),
        batch, vocab, hdim, dtype_code(hidden.dtype), vocab_offset,
        _ptr(logits), 0 if logits is None else logits.stride(0),
        _ptr(top_value), _ptr(top_index), _ptr(top_key),
        _ptr(ws), ws.numel(), _stream(hidden.device))
    _check(status, entry)


class PreparedProjection:
    """One projection call with its arguments converted once: device pointers,
    strides, sizes, dtype, workspace and stream are fixed at construction, so
    each call() only crosses the C ABI. For decode loops that call the head
    repeatedly on the same buffers (new contents each step). entry is
    "gsp_row_sparse_logits", "gsp_block_gemm_logits" or
    "gsp_dense_masked_logits"; the stream is the current one at construction."""

    def __init__(self, entry: str, hidden, weight, mask, logits=None, top_value=None, top_index=None,
                 top_key=None, vocab_offset: int = 0):
        _require_cuda(hidden, weight, mask, logits)
        lib = load()
        batch, hdim = hidden.shape
        vocab = weight.shape[0]
        ws = workspace(hidden.device, batch, vocab)
        self._keep = (hidden, weight, mask, logits, top_value, top_index, top_key, ws)
        self._entry = entry
        self._fn = getattr(lib, entry)
        self._args = (
            _ptr(hidden), hidden.stride(0), _ptr(weight), weight.stride(0),
            _ptr(mask), 0 if mask is None else mask.stride(0),
            batch, vocab, hdim, dtype_code(hidden.dtype), vocab_offset,
            _ptr(logits), 0 if logits is None else logits.stride(0),
            _ptr(top_value), _ptr(top_index), _ptr(top_key),
            _ptr(ws), ws.numel(), _stream(hidden.device))

    def __call__(self) -> None:
        status = self._fn(*self._args)
        if status:
            _check(status, self._entry)


class PreparedStep:
    """One decode step from pinned host inputs in one C-ABI call
    (gsp_row_sparse_step): the staging row host_row (pinned, the step's
    packed mask and hidden state) is copied into dev_row by the SM copy and
    the row-sparse projection runs on the views hidden / mask of dev_row;
    top_value / top_index may be pinned host tensors. Arguments are converted
    once; call(host_row) may name another pinned row of the same size."""

    def __init__(self, host_row, dev_row, hidden, weight, mask, logits=None, top_value=None, top_index=None,
                 top_key=None, vocab_offset: int = 0):
        _require_cuda(hidden, weight, mask, logits, dev_row)
        lib = load()
        batch, hdim = hidden.shape
        vocab = weight.shape[0]
        ws = workspace(hidden.device, batch, vocab)
        self._nbytes = host_row.numel() * host_row.element_size()
        self._keep = (dev_row, hidden, weight, mask, logits, top_value, top_index, top_key, ws)
        self._fn = lib.gsp_row_sparse_step
        self._tail = (
            _ptr(dev_row), _ptr(hidden), hidden.stride(0), _ptr(weight), weight.stride(0),
            _ptr(mask), 0 if mask is None else mask.stride(0),
            batch, vocab, hdim, dtype_code(hidden.dtype), vocab_offset,
            _ptr(logits), 0 if logits is None else logits.stride(0),
            _ptr(top_value), _ptr(top_index), _ptr(top_key),
            _ptr(ws), ws.numel(), _stream(hidden.device))
        self._default = host_row

    def __call__(self, host_row=None) -> None:
        row = self._default if host_row is None else host_row
        status = self._fn(_vp(row.data_ptr()), self._nbytes, *self._tail)
        if status:
            _check(status, "gsp_row_sparse_step")


class GraphStep:
    """The decode step of PreparedStep recorded once as a CUDA graph inside
    the library (gsp_step_graph_create): each call(host_row) is one
    gsp_step_graph_launch on the current stream at construction, the copy
    retargeted to host_row (a pinned row of the same size and alignment)."""

    def __init__(self, host_row, dev_row, hidden, weight, mask, logits=None, top_value=None, top_index=None,
                 top_key=None, vocab_offset: int = 0):
        _require_cuda(hidden, weight, mask, logits, dev_row)
        lib = load()
        batch, hdim = hidden.shape
        vocab = weight.shape[0]
        ws = workspace(hidden.device, batch, vocab)
        self._keep = (host_row, dev_row, hidden, weight, mask, logits, top_value, top_index, top_key, ws)
        self._lib = lib
        self._handle = _vp()
        status = lib.gsp_step_graph_create(
            ctypes.byref(self._handle), _ptr(host_row), host_row.numel() * host_row.element_size(), _ptr(dev_row),
            _ptr(hidden), hidden.stride(0), _ptr(weight), weight.stride(0),
            _ptr(mask), 0 if mask is None else mask.stride(0),
            batch, vocab, hdim, dtype_code(hidden.dtype), vocab_offset,
            _ptr(logits), 0 if logits is None else logits.stride(0),
            _ptr(top_value), _ptr(top_index), _ptr(top_key), _ptr(ws), ws.numel())
        _check(status, "gsp_step_graph_create")
        self._launch = lib.gsp_step_graph_launch
        self._stream = _stream(hidden.device)

    def __call__(self, host_row=None) -> None:
        status = self._launch(self._handle, None if host_row is None else _vp(host_row.data_ptr()), self._stream)
        if status:
            _check(status, "gsp_step_graph_launch")

    def close(self) -> None:
        if self._handle:
            self._lib.gsp_step_graph_destroy(self._handle)
            self._handle = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def row_sparse(hidden, weight, mask, logits=None, top_value=None, top_index=None, top_key=None,
               vocab_offset: int = 0) -> None:
    _projection("gsp_row_sparse_logits", hidden, weight, mask, logits, top_value, top_index,
                top_key, vocab_offset)


def block_gemm(hidden, weight, mask, logits=None, top_value=None, top_index=None, top_key=None,
               vocab_offset: int = 0) -> None:
    _projection("gsp_block_gemm_logits", hidden, weight, mask, logits, top_value, top_index,
                top_key, vocab_offset)


def dense_masked(hidden, weight, mask, logits=None, top_value=None, top_index=None, top_key=None,
                 vocab_offset: int = 0) -> None:
    _projection("gsp_dense_masked_logits", hidden, weight, mask, logits, top_value, top_index,
                top_key, vocab_offset)


# ---------------------------------------------------------------------------
# vocabulary-parallel exchange buffers and the in-kernel cross-rank top-1
# ---------------------------------------------------------------------------
def peer_exchange_alloc(world_size: int, max_batch: int) -> tuple[int, bytes]:
    """Zeroed exchange buffer on the current device: (device pointer, IPC handle)."""
    lib = load()
    nbytes = int(lib.gsp_peer_exchange_bytes(world_size, max_batch))
    if nbytes == 0:
        raise ValueError(f"bad exchange size: world {world_size}, max_batch {max_batch}")
    buf = _vp()
    handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    _check(lib.gsp_peer_exchange_alloc(nbytes, ctypes.byref(buf), handle), "gsp_peer_exchange_alloc")
    return int(buf.value), handle.raw


def peer_exchange_open(handle: bytes) -> int:
    """Maps another process's exchange buffer (same node) into this one."""
    out = _vp()
    _check(load().gsp_peer_exchange_open(ctypes.create_string_buffer(bytes(handle), IPC_HANDLE_BYTES),
                                         ctypes.byref(out)), "gsp_peer_exchange_open")
    return int(out.value)


def peer_exchange_close(ptr: int) -> None:
    _check(load().gsp_peer_exchange_close(_vp(ptr)), "gsp_peer_exchange_close")


def peer_exchange_free(ptr: int) -> None:
    _check(load().gsp_peer_exchange_free(_vp(ptr)), "gsp_peer_exchange_free")


def peer_exchange_reset(ptr: int, world_size: int, max_batch: int) -> None:
    """Zeroes this rank's own exchange buffer (synchronous)."""
    _check(load().gsp_peer_exchange_reset(_vp(ptr), world_size, max_batch), "gsp_peer_exchange_reset")


def vocab_parallel(route: str, hidden, weight, mask, peers: list[int], rank: int, max_batch: int,
                   total_vocab: int, logits=None, top_value=None, top_index=None, top_key=None,
                   vocab_offset: int = 0, wait_us: int = 0) -> None:
    """One rank's projection with the cross-rank top-1 merge in the kernel
    (gsp_vocab_parallel_logits); peers[q] is rank q's exchange buffer as
    mapped in this process, total_vocab the whole head's vocabulary, wait_us
    the longest wait for the other ranks' keys (0: 250 ms). A wait that runs
    out leaves top_index -1 for every request."""
    _require_cuda(hidden, weight, mask, logits)
    lib = load()
    batch, hdim = hidden.shape
    vocab = weight.shape[0]
    ws = workspace(hidden.device, batch, vocab)
    arr = (_vp * len(peers))(*[_vp(int(q)) for q in peers])
    status = lib.gsp_vocab_parallel_logits(
        ROUTE_CODES[route], _ptr(hidden), hidden.stride(0), _ptr(weight), weight.stride(0),
        _ptr(mask), 0 if mask is None else mask.stride(0),
        batch, vocab, hdim, dtype_code(hidden.dtype), vocab_offset,
        _ptr(logits), 0 if logits is None else logits.stride(0),
        _ptr(top_value), _ptr(top_index), _ptr(top_key),
        _ptr(ws), ws.numel(), arr, rank, len(peers), max_batch, total_vocab, wait_us, _stream(hidden.device))
    _check(status, "gsp_vocab_parallel_logits")


class PreparedVocabParallel:
    """One gsp_vocab_parallel_logits call with its arguments converted once
    (pointers, strides, sizes, the peer-buffer array, workspace and the
    current stream at construction); each call() only crosses the C ABI."""

    def __init__(self, route: str, hidden, weight, mask, peers: list[int], rank: int, max_batch: int,
                 total_vocab: int, logits=None, top_value=None, top_index=None, top_key=None,
                 vocab_offset: int = 0, wait_us: int = 0):
        _require_cuda(hidden, weight, mask, logits)
        lib = load()
        batch, hdim = hidden.shape
        vocab = weight.shape[0]
        ws = workspace(hidden.device, batch, vocab)
        arr = (_vp * len(peers))(*[_vp(int(q)) for q in peers])
        self._keep = (hidden, weight, mask, logits, top_value, top_index, top_key, ws, arr)
        self._fn = lib.gsp_vocab_parallel_logits
        self._args = (
            ROUTE_CODES[route], _ptr(hidden), hidden.stride(0), _ptr(weight), weight.stride(0),
            _ptr(mask), 0 if mask is None else mask.stride(0),
            batch, vocab, hdim, dtype_code(hidden.dtype), vocab_offset,
            _ptr(logits), 0 if logits is None else logits.stride(0),
            _ptr(top_value), _ptr(top_index), _ptr(top_key),
            _ptr(ws), ws.numel(), arr, rank, len(peers), max_batch, total_vocab, wait_us, _stream(hidden.device))

    def __call__(self) -> None:
        status = self._fn(*self._args)
        if status:
            _check(status, "gsp_vocab_parallel_logits")


def row_sparse_sample(hidden, weight, mask, seeds, offset: int, temperature: float, sample_index,
                      sample_logsumexp=None, logits=None, top_value=None, top_index=None,
                      vocab_offset: int = 0, sample_key=None, top_key=None, route: str = "row-sparse") -> None:
    """Fused sampler: Gumbel-max draw per request from softmax(logits /
    temperature) over the legal tokens, keyed by seeds[b] (uint64 stored as
    int64) and the step counter `offset`; route "row-sparse"
    (gsp_row_sparse_sample) or "block-sparse" / "dense-mask" (gsp_sample: the
    tensor-core projection with the sampler in its epilogue)."""
    _require_cuda(hidden, weight, mask, seeds, sample_index, sample_logsumexp, logits)
    lib = load()
    batch, hdim = hidden.shape
    vocab = weight.shape[0]
    ws = workspace(hidden.device, batch, vocab)
    status = lib.gsp_sample(
        ROUTE_CODES[route], _ptr(hidden), hidden.stride(0), _ptr(weight), weight.stride(0),
        _ptr(mask), 0 if mask is None else mask.stride(0),
        batch, vocab, hdim, dtype_code(hidden.dtype), vocab_offset,
        _ptr(logits), 0 if logits is None else logits.stride(0),
        float(temperature), _ptr(seeds), int(offset) & 0xFFFFFFFFFFFFFFFF,
        _ptr(sample_index), _ptr(sample_logsumexp), _ptr(sample_key), _ptr(top_value), _ptr(top_index),
        _ptr(top_key), _ptr(ws), ws.numel(), _stream(hidden.device))
    _check(status, "gsp_sample")


def merge_logsumexp(lse_parts, out) -> None:
    """gsp_merge_logsumexp: lse_parts CUDA float32 [parts, batch] -> out [batch]."""
    _require_cuda(lse_parts, out)
    status = load().gsp_merge_logsumexp(_ptr(lse_parts), lse_parts.shape[0], lse_parts.shape[1], _ptr(out),
                                        _stream(out.device))
    _check(status, "gsp_merge_logsumexp")


def row_sparse_compact(hidden, weight, mask, compact_logits, compact_ids, offsets,
                       top_value=None, top_index=None, top_key=None, vocab_offset: int = 0) -> None:
    _require_cuda(hidden, weight, mask, compact_logits, compact_ids, offsets)
    lib = load()
    batch, hdim = hidden.shape
    vocab = weight.shape[0]
    ws = workspace(hidden.device, batch, vocab)
    cap = 0 if compact_logits is None else compact_logits.numel()
    status = lib.gsp_row_sparse_compact(
        _ptr(hidden), hidden.stride(0), _ptr(weight), weight.stride(0),
        _ptr(mask), 0 if mask is None else mask.stride(0),
        batch, vocab, hdim, dtype_code(hidden.dtype), vocab_offset,
        _ptr(compact_logits), _ptr(compact_ids), cap, _ptr(offsets),
        _ptr(top_value), _ptr(top_index), _ptr(top_key),
        _ptr(ws), ws.numel(), _stream(hidden.device))
    _check(status, "gsp_row_sparse_compact")


def ids_to_bitmask(ids: torch.Tensor, vocab: int, bitmask: torch.Tensor, stats: torch.Tensor) -> None:
    _require_cuda(ids, bitmask, stats)
    status = load().gsp_ids_to_bitmask(_ptr(ids), ids.numel(), vocab, _ptr(bitmask), _ptr(stats),
                                       _stream(ids.device))
    _check(status, "gsp_ids_to_bitmask")


def mask_stats(mask: torch.Tensor, vocab: int, legal_counts=None, full_words=None,
               active_tiles=None) -> None:
    _require_cuda(mask)
    batch = mask.shape[0]
    status = load().gsp_mask_stats(_ptr(mask), mask.stride(0), batch, vocab, _ptr(legal_counts),
                                   _ptr(full_words), _ptr(active_tiles), _stream(mask.device))
    _check(status, "gsp_mask_stats")


def top1_from_keys(keys: torch.Tensor, top_value=None, top_index=None) -> None:
    _require_cuda(keys)
    status = load().gsp_top1_from_keys(_ptr(keys), keys.numel(), _ptr(top_value), _ptr(top_index),
                                       _stream(keys.device))
    _check(status, "gsp_top1_from_keys")


# ---------------------------------------------------------------------------
# device-side route choice
# ---------------------------------------------------------------------------
def route_cost(cost: dict | None) -> RouteCost | None:
    """RouteCost from a dict of gsp_route_cost fields (missing fields take the
    library defaults); None stays None (the library's B200 defaults)."""
    if cost is None:
        return None
    c = RouteCost()
    load().gsp_default_route_cost(ctypes.byref(c))
    for name, value in cost.items():
        if name not in dict(RouteCost._fields_):
            raise ValueError(f"unknown route cost field {name!r}")
        setattr(c, name, float(value))
    return c


def default_route_cost() -> dict:
    """The library's built-in B200 route cost model (gsp_default_route_cost)."""
    c = RouteCost()
    load().gsp_default_route_cost(ctypes.byref(c))
    return {name: getattr(c, name) for name, _ in RouteCost._fields_}


def choose_route_code(batch: int, vocab: int, hidden_dim: int, elem_bytes: int, legal_total: int,
                      active_tiles: int, cost: dict | None = None) -> int:
    """The library's route choice for given statistics (gsp_choose_route, host)."""
    c = route_cost(cost)
    status = load().gsp_choose_route(batch, vocab, hidden_dim, elem_bytes, legal_total, active_tiles,
                                     None if c is None else ctypes.byref(c))
    if status < 0:
        _check(status, "gsp_choose_route")
    return status


def adaptive(hidden, weight, mask, logits=None, top_value=None, top_index=None, route_out=None,
             cost: dict | None = None) -> int:
    """gsp_adaptive_logits: route chosen on the device. Returns the route code
    (eager calls) or -1 (stream being captured: a conditional node chooses at
    every replay; route_out, an int32 CUDA tensor, then holds it)."""
    _require_cuda(hidden, weight, mask, logits)
    lib = load()
    batch, hdim = hidden.shape
    vocab = weight.shape[0]
    ws = workspace(hidden.device, batch, vocab)
    c = route_cost(cost)
    host_route = ctypes.c_int32(-1)
    status = lib.gsp_adaptive_logits(
        _ptr(hidden), hidden.stride(0), _ptr(weight), weight.stride(0), _ptr(mask),
        0 if mask is None else mask.stride(0), batch, vocab, hdim, dtype_code(hidden.dtype),
        _ptr(logits), 0 if logits is None else logits.stride(0), _ptr(top_value), _ptr(top_index),
        None if c is None else ctypes.byref(c), _ptr(route_out), ctypes.byref(host_route),
        _ptr(ws), ws.numel(), _stream(hidden.device))
    _check(status, "gsp_adaptive_logits")
    return host_route.value


# ---------------------------------------------------------------------------
# lane grouping by density class
# ---------------------------------------------------------------------------
GROUP_PLAN_HEADER = 16
GROUP_MAX_BATCH = 256


def group_plan(mask, vocab: int, hidden_dim: int, elem_bytes: int, with_logits: bool, plan,
               cost: dict | None = None) -> None:
    """gsp_group_plan into `plan` (CUDA int32, gsp_group_plan_words(batch))."""
    _require_cuda(mask, plan)
    c = route_cost(cost)
    batch = mask.shape[0]
    status = load().gsp_group_plan(_ptr(mask), mask.stride(0), batch, vocab, hidden_dim, elem_bytes,
                                   1 if with_logits else 0, None if c is None else ctypes.byref(c), _ptr(plan),
                                   _stream(mask.device))
    _check(status, "gsp_group_plan")


def gather_rows(src, rows, dst, n: int | None = None) -> None:
    """dst[i] = src[rows[i]] for i < n (rows: CUDA int32; 2-D src/dst, or 1-D
    for one element per row)."""
    _require_cuda(src, rows, dst)
    n = rows.numel() if n is None else n
    row_bytes = (src.shape[1] if src.ndim == 2 else 1) * src.element_size()
    status = load().gsp_gather_rows(_ptr(src), src.stride(0) * src.element_size(), _ptr(rows), n, row_bytes,
                                    _ptr(dst), dst.stride(0) * dst.element_size(), _stream(src.device))
    _check(status, "gsp_gather_rows")


_scratch: dict[tuple[int, int], torch.Tensor] = {}


def _grouped_scratch(device: torch.device, need: int) -> torch.Tensor:
    dev_index = device.index if device.index is not None else torch.cuda.current_device()
    key = (dev_index, torch.cuda.current_stream(device).cuda_stream)
    with _ws_lock:
        buf = _scratch.get(key)
        if buf is None or buf.numel() < need:
            buf = torch.empty(max(need, 2 * (0 if buf is None else buf.numel())), dtype=torch.uint8, device=device)
            _scratch[key] = buf
        return buf


def grouped(hidden, weight, mask, logits=None, top_value=None, top_index=None, cost: dict | None = None) -> list[int]:
    """gsp_grouped_logits; returns the plan header [k, route A, route B, best
    single route, single ns, split ns, 0, 0] (waits for the plan)."""
    _require_cuda(hidden, weight, mask, logits)
    lib = load()
    batch, hdim = hidden.shape
    vocab = weight.shape[0]
    ws = workspace(hidden.device, batch, vocab)
    scratch = _grouped_scratch(hidden.device, int(lib.gsp_grouped_scratch_bytes(batch, vocab, hdim,
                                                                                 1 if logits is not None else 0)))
    c = route_cost(cost)
    hdr = (_i32 * 8)()
    status = lib.gsp_grouped_logits(
        _ptr(hidden), hidden.stride(0), _ptr(weight), weight.stride(0), _ptr(mask), mask.stride(0),
        batch, vocab, hdim, dtype_code(hidden.dtype), _ptr(logits), 0 if logits is None else logits.stride(0),
        _ptr(top_value), _ptr(top_index), None if c is None else ctypes.byref(c), hdr,
        _ptr(scratch), scratch.numel(), _ptr(ws), ws.numel(), _stream(hidden.device))
    _check(status, "gsp_grouped_logits")
    return list(hdr)


def copy_bytes(dst: torch.Tensor, src: torch.Tensor, nbytes: int | None = None) -> None:
    """gsp_copy_bytes on the current stream of whichever tensor is on a CUDA
    device: an SM-driven copy (pinned host tensors included)."""
    n = src.numel() * src.element_size() if nbytes is None else nbytes
    dev = dst.device if dst.device.type == "cuda" else src.device
    status = load().gsp_copy_bytes(_ptr(dst), _ptr(src), n, _stream(dev))
    _check(status, "gsp_copy_bytes")
