"""ctypes binding of ``libsparseconv_b200.so`` (the C ABI declared in
``include/sparseconv_b200.h``) plus the tensor-level helpers the front end calls.

There is no CPU fallback: if the library is missing, or a tensor is not on a CUDA device,
every call raises. Outputs are allocated from torch's caching allocator and every launch
goes to ``torch.cuda.current_stream()``.

Device-side problems (coordinates out of range, a full table, a kernel wait limit) are
OR-ed into a per-device int32 status word. After each op the word is copied
asynchronously to pinned host memory; the next op on that device (or an explicit
``check_errors()``) raises ``RuntimeError`` if a bit is set. With the environment variable
``SPARSECONV_SYNC_CHECK=1`` each op synchronises and checks at once.
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional, Sequence, Tuple

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libsparseconv_b200.so")

SPCONV_OK, SPCONV_ERR_ARG, SPCONV_ERR_CUDA, SPCONV_ERR_UNSUPPORTED = 0, 1, 2, 3
STATUS_COORD_RANGE, STATUS_TABLE_FULL, STATUS_DUPLICATE, STATUS_WAIT_TIMEOUT = 1, 2, 4, 8
DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
KERNEL_AUTO, KERNEL_SIMT, KERNEL_TCGEN05 = 0, 1, 2
NOALLOC_MAX_COORDS = 262144   # SPCONV_NOALLOC_MAX_COORDS

_c_i64, _c_int, _c_void_p = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p

# name -> (restype, argtypes); the order mirrors include/sparseconv_b200.h
SIGNATURES = {
    "spconv_abi_version": (_c_int, []),
    "spconv_last_error": (ctypes.c_char_p, []),
    "spconv_hashmap_capacity": (_c_i64, [_c_i64]),
    "spconv_mask_words": (_c_int, [_c_int]),
    "spconv_neighbor_map_workspace_bytes": (_c_i64, [_c_i64, _c_int, _c_int, _c_int, _c_int]),
    "spconv_build_submanifold_neighbor_map": (_c_int, [
        _c_void_p, _c_i64, _c_int, _c_int, _c_int, _c_int,
        _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
        _c_void_p, _c_i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "spconv_submanifold_conv_forward": (_c_int, [
        _c_void_p, _c_int, _c_i64, _c_int, _c_void_p, _c_void_p, _c_int, _c_int,
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "spconv_submanifold_conv_forward_ex": (_c_int, [
        _c_void_p, _c_int, _c_i64, _c_int, _c_void_p, _c_void_p, _c_int, _c_int,
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int]),
    "spconv_conv_splitk_workspace_bytes": (_c_i64, [_c_i64, _c_int]),
    "spconv_submanifold_conv_forward_splitk": (_c_int, [
        _c_void_p, _c_int, _c_i64, _c_int, _c_void_p, _c_void_p, _c_int, _c_int,
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_i64, _c_void_p, _c_void_p, _c_void_p]),
    "spconv_build_submanifold_neighbor_map_noalloc": (_c_int, [
        _c_void_p, _c_i64, _c_int, _c_int, _c_int, _c_int,
        _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "spconv_neighbor_map_2d_workspace_bytes": (_c_i64, [_c_i64, _c_int, _c_int, _c_int]),
    "spconv_build_submanifold_neighbor_map_2d": (_c_int, [
        _c_void_p, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
        _c_void_p, _c_i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "spconv_from_dense_workspace_bytes": (_c_i64, [_c_int, _c_int, _c_int, _c_int]),
    "spconv_from_dense": (_c_int, [
        _c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_i64, _c_void_p,
        _c_void_p, _c_void_p, _c_i64, _c_int, _c_void_p]),
    "spconv_to_dense": (_c_int, [
        _c_void_p, _c_int, _c_void_p, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
        _c_void_p, _c_void_p, _c_void_p]),
    "spconv_hashmap_insert": (_c_int, [
        _c_void_p, _c_void_p, _c_i64, _c_int, _c_int, _c_void_p, _c_void_p, _c_i64, _c_void_p, _c_void_p]),
    "spconv_hashmap_lookup": (_c_int, [
        _c_void_p, _c_void_p, _c_i64, _c_int, _c_int, _c_void_p, _c_void_p, _c_i64, _c_void_p]),
    "spconv_submanifold_conv_backward_input": (_c_int, [
        _c_void_p, _c_int, _c_i64, _c_int, _c_void_p, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p,
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "spconv_transpose_neighbor_map": (_c_int, [
        _c_void_p, _c_i64, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "spconv_weight_grad_workspace_bytes": (_c_i64, [_c_i64, _c_int]),
    "spconv_submanifold_conv_weight_grad": (_c_int, [
        _c_void_p, _c_void_p, _c_int, _c_i64, _c_int, _c_int, _c_int,
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_i64, _c_void_p, _c_void_p]),
    "spconv_set_wait_limit_ns": (ctypes.c_uint64, [ctypes.c_uint64]),
    "spconv_stage_timing": (_c_int, [_c_int]),
    "spconv_stage_times_ms": (_c_int, [_c_void_p, _c_void_p, _c_int]),
}

STAGES = ("memset", "insert", "map", "order", "conv")

_lib = None
_lock = threading.Lock()


def load_library(path: Optional[str] = None) -> ctypes.CDLL:
    """Load the CUDA library (once). Raises RuntimeError if it has not been built."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise RuntimeError(
            f"sparseconv CUDA library not found at {p}; build it with "
            "`python sparse-conv_b200/build.py` (there is no CPU fallback)")
    lib = ctypes.CDLL(p)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.spconv_abi_version() != 1:
        raise RuntimeError("sparseconv CUDA library ABI version mismatch")
    if path is None:
        _lib = lib
    return lib


def _raise(rc: int, what: str) -> None:
    msg = load_library().spconv_last_error().decode(errors="replace")
    if rc == SPCONV_ERR_ARG:
        raise ValueError(f"{what}: {msg}")
    if rc == SPCONV_ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg}")


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "sparseconv runs on CUDA devices only (no CPU fallback); got a tensor on "
                f"{t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    return dev


# ---------------------------------------------------------------------------------------
# Device status word and deferred checks.
# ---------------------------------------------------------------------------------------
class _DeviceStatus:
    def __init__(self, device: torch.device):
        self.device = device
        self.word = torch.zeros(1, dtype=torch.int32, device=device)
        self.host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.event = torch.cuda.Event()
        self.pending = False


_status = {}


def status_word(device: torch.device) -> _DeviceStatus:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _status.get(idx)
    if st is None:
        with _lock:
            st = _status.get(idx)
            if st is None:
                st = _DeviceStatus(torch.device("cuda", idx))
                _status[idx] = st
    return st


def describe_status(bits: int) -> str:
    parts = []
    if bits & STATUS_COORD_RANGE:
        parts.append("a coordinate lies outside the spatial shape [0,N)x[0,W)x[0,H)x[0,D)")
    if bits & STATUS_TABLE_FULL:
        parts.append("the coordinate hash table overflowed")
    if bits & STATUS_WAIT_TIMEOUT:
        parts.append("a kernel-internal wait reached its time limit")
    return "; ".join(parts)


_FATAL_BITS = STATUS_COORD_RANGE | STATUS_TABLE_FULL | STATUS_WAIT_TIMEOUT


def _inspect(st: _DeviceStatus) -> None:
    bits = int(st.host.item())
    st.pending = False
    if bits & _FATAL_BITS:
        st.word.zero_()
        raise RuntimeError(f"sparseconv device error: {describe_status(bits)} (status bits {bits:#x})")


def after_launch(device: torch.device) -> None:
    """Queue the status read-back of this op; check at once if SPARSECONV_SYNC_CHECK=1.

    Skipped while the stream is being captured into a CUDA graph (call ``check_errors``
    after replays instead)."""
    if torch.cuda.is_current_stream_capturing():
        return
    st = status_word(device)
    stream = torch.cuda.current_stream(device)
    st.host.copy_(st.word, non_blocking=True)
    st.event.record(stream)
    st.pending = True
    if os.environ.get("SPARSECONV_SYNC_CHECK", "0") == "1":
        st.event.synchronize()
        _inspect(st)


def before_launch(device: torch.device) -> None:
    """Raise for an error found by an earlier op on this device, if its read-back landed."""
    if torch.cuda.is_current_stream_capturing():
        return
    st = status_word(device)
    if st.pending and st.event.query():
        _inspect(st)


def check_errors(device: Optional[torch.device] = None) -> int:
    """Synchronise with the device's status read-back and raise on an error.

    Returns the status bits seen (duplicate coordinates are reported, not raised).
    """
    devs = [status_word(device)] if device is not None else list(_status.values())
    bits = 0
    for st in devs:
        if st.pending:
            st.event.synchronize()
        torch.cuda.synchronize(st.device)
        st.host.copy_(st.word)
        bits |= int(st.host.item())
        _inspect(st)
    return bits


def reset_status(device: Optional[torch.device] = None) -> None:
    for st in ([status_word(device)] if device is not None else list(_status.values())):
        st.word.zero_()
        st.pending = False


# ---------------------------------------------------------------------------------------
# Tensor-level calls.
# ---------------------------------------------------------------------------------------
def mask_words(kernel_volume: int) -> int:
    return int(load_library().spconv_mask_words(int(kernel_volume)))


def hashmap_capacity(num_coords: int) -> int:
    return int(load_library().spconv_hashmap_capacity(int(num_coords)))


def workspace_bytes(num_coords: int, batch: int, W: int, H: int, D: int) -> int:
    return int(load_library().spconv_neighbor_map_workspace_bytes(int(num_coords), batch, W, H, D))


def build_neighbor_map(coords: torch.Tensor, batch: int, W: int, H: int, D: int,
                       kernel_size: Sequence[int], dilation: Sequence[int],
                       workspace: Optional[torch.Tensor] = None,
                       ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Kernel map of ``coords`` ([M,4] int32 on CUDA): (neighbor_map [M,V] int32,
    masks [M,ceil(V/32)] int32 bit patterns, order [M] int32)."""
    lib = load_library()
    dev = _require_cuda(coords)
    if coords.dtype != torch.int32 or coords.dim() != 2 or coords.shape[1] != 4:
        raise ValueError("coords must be an [M, 4] int32 tensor")
    if not coords.is_contiguous():
        raise ValueError("coords must be contiguous")
    Kw, Kh, Kd = (int(k) for k in kernel_size)
    Dw, Dh, Dd = (int(d) for d in dilation)
    M = int(coords.shape[0])
    V = Kw * Kh * Kd
    MW = max(1, mask_words(V))
    nbr = torch.empty((M, V), dtype=torch.int32, device=dev)
    masks = torch.empty((M, MW), dtype=torch.int32, device=dev)
    order = torch.empty((M,), dtype=torch.int32, device=dev)
    if M == 0:
        return nbr, masks, order
    need = workspace_bytes(M, batch, W, H, D)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty((need,), dtype=torch.uint8, device=dev)
    before_launch(dev)
    st = status_word(dev)
    rc = lib.spconv_build_submanifold_neighbor_map(
        coords.data_ptr(), M, int(batch), int(W), int(H), int(D), Kw, Kh, Kd, Dw, Dh, Dd,
        workspace.data_ptr(), need, nbr.data_ptr(), masks.data_ptr(), order.data_ptr(),
        st.word.data_ptr(), _stream_ptr(dev))
    if rc != SPCONV_OK:
        _raise(rc, "spconv_build_submanifold_neighbor_map")
    return nbr, masks, order


def build_neighbor_map_2d(coords: torch.Tensor, batch: int, W: int, H: int,
                          kernel_size: Sequence[int], dilation: Sequence[int],
                          ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """2-D kernel map of ``coords`` ([M,3] int32 (b, x, y) on CUDA): (neighbor_map [M, Kw*Kh]
    int32, masks, order), the map of the reference's
    ``hashmap_build_submanifold_conv2d_neighbor_map_cuda_naive`` (neighbor_map.cu:10-111)."""
    lib = load_library()
    dev = _require_cuda(coords)
    if coords.dtype != torch.int32 or coords.dim() != 2 or coords.shape[1] != 3:
        raise ValueError("coords must be an [M, 3] int32 tensor")
    if not coords.is_contiguous():
        raise ValueError("coords must be contiguous")
    Kw, Kh = (int(k) for k in kernel_size)
    Dw, Dh = (int(d) for d in dilation)
    M = int(coords.shape[0])
    V = Kw * Kh
    nbr = torch.empty((M, V), dtype=torch.int32, device=dev)
    masks = torch.empty((M, max(1, mask_words(V))), dtype=torch.int32, device=dev)
    order = torch.empty((M,), dtype=torch.int32, device=dev)
    if M == 0:
        return nbr, masks, order
    need = int(lib.spconv_neighbor_map_2d_workspace_bytes(M, int(batch), int(W), int(H)))
    if need < 0:
        raise ValueError("invalid 2-D map arguments")
    workspace = torch.empty((need,), dtype=torch.uint8, device=dev)
    before_launch(dev)
    st = status_word(dev)
    rc = lib.spconv_build_submanifold_neighbor_map_2d(
        coords.data_ptr(), M, int(batch), int(W), int(H), Kw, Kh, Dw, Dh, workspace.data_ptr(), need,
        nbr.data_ptr(), masks.data_ptr(), order.data_ptr(), st.word.data_ptr(), _stream_ptr(dev))
    if rc != SPCONV_OK:
        _raise(rc, "spconv_build_submanifold_neighbor_map_2d")
    return nbr, masks, order


def conv_forward(feats: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
                 nbr: torch.Tensor, masks: Optional[torch.Tensor], order: Optional[torch.Tensor],
                 kernel: int = KERNEL_AUTO, out: Optional[torch.Tensor] = None,
                 split: bool = False) -> torch.Tensor:
    """out[i] = bias + sum_v feats[nbr[i,v]] @ weight[:, v, :]^T over valid neighbours.

    ``weight`` is [Co, V, Ci] (or [Co, Kw, Kh, Kd, Ci]) in the dtype of ``feats``. ``split``
    runs the split-K variant (``spconv_submanifold_conv_forward_splitk``: the heaviest tiles'
    offsets spread over two CTAs, fp32 partials in a workspace from torch's allocator).
    """
    lib = load_library()
    dev = _require_cuda(feats, weight, bias, nbr, masks, order)
    if feats.dtype not in DTYPE_CODES:
        raise TypeError(f"unsupported feature dtype {feats.dtype}")
    if not feats.is_contiguous():
        raise ValueError("feats must be contiguous")
    M, Ci = int(feats.shape[0]), int(feats.shape[1])
    Co = int(weight.shape[0])
    V = int(nbr.shape[1]) if nbr.dim() == 2 else 0
    if nbr.shape[0] != M:
        raise ValueError(f"neighbor map has {nbr.shape[0]} rows for {M} feature rows")
    w = weight.reshape(Co, V, Ci)
    if w.dtype != feats.dtype:
        w = w.to(feats.dtype)
    w = w.contiguous()
    b = None
    if bias is not None:
        b = bias.to(feats.dtype).contiguous()
        if b.numel() != Co:
            raise ValueError(f"bias has {b.numel()} entries for {Co} output channels")
    nb = nbr.view(torch.int32) if nbr.dtype == torch.uint32 else nbr
    if nb.dtype != torch.int32 or not nb.is_contiguous():
        raise ValueError("neighbor map must be a contiguous [M, V] int32/uint32 tensor")
    mk = None
    if masks is not None:
        mk = masks.view(torch.int32) if masks.dtype == torch.uint32 else masks
        if mk.dtype != torch.int32 or mk.shape[0] != M or not mk.is_contiguous():
            raise ValueError("masks must be a contiguous [M, ceil(V/32)] 32-bit tensor")
    od = None
    if order is not None:
        if order.dtype != torch.int32 or order.numel() != M or not order.is_contiguous():
            raise ValueError("order must be a contiguous [M] int32 tensor")
        od = order
    if out is None:
        out = torch.empty((M, Co), dtype=feats.dtype, device=dev)
    if M == 0:
        return out
    before_launch(dev)
    st = status_word(dev)
    if split:
        need = int(lib.spconv_conv_splitk_workspace_bytes(M, Co))
        ws = torch.empty((need,), dtype=torch.uint8, device=dev)
        rc = lib.spconv_submanifold_conv_forward_splitk(
            feats.data_ptr(), DTYPE_CODES[feats.dtype], M, Ci, w.data_ptr(),
            None if b is None else b.data_ptr(), Co, V, nb.data_ptr(),
            None if mk is None else mk.data_ptr(), None if od is None else od.data_ptr(),
            ws.data_ptr(), need, out.data_ptr(), st.word.data_ptr(), _stream_ptr(dev))
        if rc != SPCONV_OK:
            _raise(rc, "spconv_submanifold_conv_forward_splitk")
        return out
    rc = lib.spconv_submanifold_conv_forward_ex(
        feats.data_ptr(), DTYPE_CODES[feats.dtype], M, Ci, w.data_ptr(),
        None if b is None else b.data_ptr(), Co, V, nb.data_ptr(),
        None if mk is None else mk.data_ptr(), None if od is None else od.data_ptr(),
        out.data_ptr(), st.word.data_ptr(), _stream_ptr(dev), int(kernel))
    if rc != SPCONV_OK:
        _raise(rc, "spconv_submanifold_conv_forward")
    return out


def dense_to_sparse(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """(indices [M,4] int32 (b,x,y,z), features [M,C]) of the voxels of a channels-last dense
    [B, W, H, D, C] CUDA tensor with any non-zero channel, in (b, x, y, z) order. Reads the
    number of active voxels back to the host (one synchronisation) to size the outputs."""
    lib = load_library()
    dev = _require_cuda(x)
    if x.dtype not in DTYPE_CODES or x.dim() != 5:
        raise ValueError("expected a [B, W, H, D, C] float32/float16/bfloat16 tensor")
    x = x.contiguous()
    B, W, H, D, C = (int(v) for v in x.shape)
    if B * W * H * D == 0 or C == 0:
        return (torch.empty((0, 4), dtype=torch.int32, device=dev),
                torch.empty((0, C), dtype=x.dtype, device=dev))
    need = int(lib.spconv_from_dense_workspace_bytes(B, W, H, D))
    if need <= 0:
        raise ValueError("dense tensor too large")
    ws = torch.empty((need,), dtype=torch.uint8, device=dev)
    count = torch.zeros((1,), dtype=torch.int64, device=dev)
    stream = _stream_ptr(dev)
    rc = lib.spconv_from_dense(x.data_ptr(), DTYPE_CODES[x.dtype], B, W, H, D, C, ws.data_ptr(), need,
                               count.data_ptr(), None, None, 0, 0, stream)
    if rc != SPCONV_OK:
        _raise(rc, "spconv_from_dense")
    M = int(count.item())
    indices = torch.empty((M, 4), dtype=torch.int32, device=dev)
    feats = torch.empty((M, C), dtype=x.dtype, device=dev)
    rc = lib.spconv_from_dense(x.data_ptr(), DTYPE_CODES[x.dtype], B, W, H, D, C, ws.data_ptr(), need,
                               count.data_ptr(), indices.data_ptr(), feats.data_ptr(), M, 1, stream)
    if rc != SPCONV_OK:
        _raise(rc, "spconv_from_dense")
    return indices, feats


def sparse_to_dense(feats: torch.Tensor, indices: torch.Tensor, batch: int, spatial: Sequence[int],
                    channels_first: bool = True) -> torch.Tensor:
    """Zero dense tensor [B, C, W, H, D] (or [B, W, H, D, C]) with the rows of ``feats`` at
    ``indices`` ([M,4] int32 (b,x,y,z))."""
    lib = load_library()
    dev = _require_cuda(feats, indices)
    if feats.dtype not in DTYPE_CODES:
        raise TypeError(f"unsupported feature dtype {feats.dtype}")
    feats = feats.contiguous()
    idx = indices.to(torch.int32).contiguous()
    M, C = int(feats.shape[0]), int(feats.shape[1])
    W, H, D = (int(v) for v in spatial)
    shape = (batch, C, W, H, D) if channels_first else (batch, W, H, D, C)
    out = torch.empty(shape, dtype=feats.dtype, device=dev)
    before_launch(dev)
    st = status_word(dev)
    rc = lib.spconv_to_dense(feats.data_ptr(), DTYPE_CODES[feats.dtype], idx.data_ptr(), M, C, int(batch), W, H, D,
                             1 if channels_first else 0, out.data_ptr(), st.word.data_ptr(), _stream_ptr(dev))
    if rc != SPCONV_OK:
        _raise(rc, "spconv_to_dense")
    return out


_BITS = {torch.uint32: 32, torch.int32: 32, torch.uint64: 64, torch.int64: 64}


def _table_args(table_keys: torch.Tensor, table_values: torch.Tensor, keys: torch.Tensor):
    if table_keys.dtype not in _BITS or table_values.dtype not in _BITS:
        raise TypeError("table keys / values must be 32- or 64-bit integer tensors")
    if keys.dtype != table_keys.dtype:
        raise TypeError(f"keys dtype {keys.dtype} differs from the table's {table_keys.dtype}")
    if not (table_keys.is_contiguous() and table_values.is_contiguous()):
        raise ValueError("table tensors must be contiguous")
    if table_keys.numel() != table_values.numel() or table_keys.numel() == 0:
        raise ValueError("table keys and values must have the same, non-zero length")
    return int(table_keys.numel()), _BITS[table_keys.dtype], _BITS[table_values.dtype]


def hashmap_insert(table_keys: torch.Tensor, table_values: torch.Tensor, keys: torch.Tensor,
                   values: torch.Tensor) -> None:
    """hashmap_insert_cuda (hash.cu:8-71): insert keys -> values into the caller's table."""
    lib = load_library()
    dev = _require_cuda(table_keys, table_values, keys, values)
    cap, kb, vb = _table_args(table_keys, table_values, keys)
    if values.dtype != table_values.dtype or values.numel() != keys.numel():
        raise ValueError("values must match the table's value dtype and the number of keys")
    k, v = keys.contiguous(), values.contiguous()
    before_launch(dev)
    st = status_word(dev)
    rc = lib.spconv_hashmap_insert(table_keys.data_ptr(), table_values.data_ptr(), cap, kb, vb, k.data_ptr(),
                                   v.data_ptr(), int(k.numel()), st.word.data_ptr(), _stream_ptr(dev))
    if rc != SPCONV_OK:
        _raise(rc, "spconv_hashmap_insert")
    after_launch(dev)


def hashmap_lookup(table_keys: torch.Tensor, table_values: torch.Tensor, keys: torch.Tensor) -> torch.Tensor:
    """hashmap_lookup_cuda (hash.cu:73-146): values of keys (all ones if absent)."""
    lib = load_library()
    dev = _require_cuda(table_keys, table_values, keys)
    cap, kb, vb = _table_args(table_keys, table_values, keys)
    k = keys.contiguous()
    out = torch.empty((k.numel(),), dtype=table_values.dtype, device=dev)
    rc = lib.spconv_hashmap_lookup(table_keys.data_ptr(), table_values.data_ptr(), cap, kb, vb, k.data_ptr(),
                                   out.data_ptr(), int(k.numel()), _stream_ptr(dev))
    if rc != SPCONV_OK:
        _raise(rc, "spconv_hashmap_lookup")
    return out


def conv_backward_input(grad_out: torch.Tensor, weight: torch.Tensor, nbr: torch.Tensor,
                        masks: Optional[torch.Tensor], order: Optional[torch.Tensor],
                        nbr_t: Optional[torch.Tensor] = None, masks_t: Optional[torch.Tensor] = None
                        ) -> torch.Tensor:
    """grad_in[j] = sum over (i, v) with nbr[i, v] = j of grad_out[i] @ weight[:, v, :], for
    weight [Co, V, Ci] (or [Co, Kw, Kh, Kd, Ci]). Odd V reads ``nbr`` with the offsets reversed;
    even V needs ``nbr_t`` / ``masks_t`` from ``transpose_neighbor_map``."""
    lib = load_library()
    dev = _require_cuda(grad_out, weight, nbr, masks, order, nbr_t, masks_t)
    if grad_out.dtype not in DTYPE_CODES:
        raise TypeError(f"unsupported dtype {grad_out.dtype}")
    g = grad_out.contiguous()
    M, Co = int(g.shape[0]), int(g.shape[1])
    nb = nbr.view(torch.int32) if nbr.dtype == torch.uint32 else nbr
    V = int(nb.shape[1])
    Ci = int(weight.shape[-1])
    if int(weight.shape[0]) != Co:
        raise ValueError(f"weight has {weight.shape[0]} output channels, grad_out {Co}")
    if V % 2 == 0 and nbr_t is None:
        raise ValueError("an even kernel volume needs the transposed map (transpose_neighbor_map)")
    w_t = weight.reshape(Co, V, Ci).permute(2, 1, 0).to(g.dtype).contiguous()      # [Ci, V, Co]

    def i32(t):
        return None if t is None else (t.view(torch.int32) if t.dtype == torch.uint32 else t)

    def ptr(t):
        return None if t is None else t.data_ptr()
    out = torch.empty((M, Ci), dtype=g.dtype, device=dev)
    if M == 0:
        return out
    before_launch(dev)
    st = status_word(dev)
    rc = lib.spconv_submanifold_conv_backward_input(
        g.data_ptr(), DTYPE_CODES[g.dtype], M, Co, w_t.data_ptr(), Ci, V, nb.data_ptr(), ptr(i32(masks)),
        ptr(order), ptr(i32(nbr_t)), ptr(i32(masks_t)), out.data_ptr(), st.word.data_ptr(), _stream_ptr(dev))
    if rc != SPCONV_OK:
        _raise(rc, "spconv_submanifold_conv_backward_input")
    return out


def transpose_neighbor_map(nbr: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """(nbr_t, masks_t): nbr_t[j, v] = i where nbr[i, v] = j (-1 if none), and its offset masks."""
    lib = load_library()
    dev = _require_cuda(nbr)
    nb = nbr.view(torch.int32) if nbr.dtype == torch.uint32 else nbr
    if nb.dtype != torch.int32 or nb.dim() != 2 or not nb.is_contiguous():
        raise ValueError("neighbor map must be a contiguous [M, V] int32/uint32 tensor")
    M, V = int(nb.shape[0]), int(nb.shape[1])
    nbr_t = torch.empty((M, V), dtype=torch.int32, device=dev)
    masks_t = torch.empty((M, mask_words(V)), dtype=torch.int32, device=dev)
    if M == 0:
        return nbr_t, masks_t
    before_launch(dev)
    st = status_word(dev)
    rc = lib.spconv_transpose_neighbor_map(nb.data_ptr(), M, V, nbr_t.data_ptr(), masks_t.data_ptr(),
                                           st.word.data_ptr(), _stream_ptr(dev))
    if rc != SPCONV_OK:
        _raise(rc, "spconv_transpose_neighbor_map")
    return nbr_t, masks_t


def conv_weight_grad(feats: torch.Tensor, grad_out: torch.Tensor, nbr: torch.Tensor,
                     order: Optional[torch.Tensor], with_bias: bool = True,
                     masks: Optional[torch.Tensor] = None
                     ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """(grad_weight [Co, V, Ci] fp32, grad_bias [Co] fp32 or None) of the submanifold conv:
    grad_weight[co, v, ci] = sum_i grad_out[i, co] * feats[nbr[i, v], ci]."""
    lib = load_library()
    dev = _require_cuda(feats, grad_out, nbr, order, masks)
    if feats.dtype not in DTYPE_CODES:
        raise TypeError(f"unsupported feature dtype {feats.dtype}")
    if grad_out.dtype != feats.dtype:
        raise TypeError(f"grad_out dtype {grad_out.dtype} differs from feats dtype {feats.dtype}")
    if not (feats.is_contiguous() and grad_out.is_contiguous()):
        raise ValueError("feats and grad_out must be contiguous")
    nb = nbr.view(torch.int32) if nbr.dtype == torch.uint32 else nbr
    if nb.dtype != torch.int32 or nb.dim() != 2 or not nb.is_contiguous():
        raise ValueError("neighbor map must be a contiguous [M, V] int32/uint32 tensor")
    M, Ci = int(feats.shape[0]), int(feats.shape[1])
    Co, V = int(grad_out.shape[1]), int(nb.shape[1])
    if grad_out.shape[0] != M or nb.shape[0] != M:
        raise ValueError("feats, grad_out and neighbor map must have the same number of rows")
    if order is not None and (order.dtype != torch.int32 or order.numel() != M or not order.is_contiguous()):
        raise ValueError("order must be a contiguous [M] int32 tensor")
    mk = None
    if masks is not None:
        mk = masks.view(torch.int32) if masks.dtype == torch.uint32 else masks
        if mk.dtype != torch.int32 or mk.shape[0] != M or not mk.is_contiguous():
            raise ValueError("masks must be a contiguous [M, ceil(V/32)] 32-bit tensor")
    gw = torch.empty((Co, V, Ci), dtype=torch.float32, device=dev)
    gb = torch.empty((Co,), dtype=torch.float32, device=dev) if with_bias else None
    ws_bytes = int(lib.spconv_weight_grad_workspace_bytes(M, V))
    ws = torch.empty((max(ws_bytes, 16) + 15) // 16 * 16, dtype=torch.uint8, device=dev)
    before_launch(dev)
    st = status_word(dev)
    rc = lib.spconv_submanifold_conv_weight_grad(
        feats.data_ptr(), grad_out.data_ptr(), DTYPE_CODES[feats.dtype], M, Ci, Co, V, nb.data_ptr(),
        None if mk is None else mk.data_ptr(), None if order is None else order.data_ptr(), gw.data_ptr(),
        None if gb is None else gb.data_ptr(), ws.data_ptr(), ws.numel(), st.word.data_ptr(), _stream_ptr(dev))
    if rc != SPCONV_OK:
        _raise(rc, "spconv_submanifold_conv_weight_grad")
    return gw, gb


def set_wait_limit_ns(limit_ns: int) -> int:
    """Time limit of the pipeline waits inside the tensor-core conv kernels launched from now
    on (process-wide; 0 restores the 2 s default). Returns the previous limit. A kernel whose
    wait reaches it abandons its work and reports SPCONV_STATUS_WAIT_TIMEOUT."""
    return int(load_library().spconv_set_wait_limit_ns(int(limit_ns)))


def stage_timing(max_calls: int) -> None:
    """Start (max_calls > 0) or stop (0) per-stage device timing inside the library."""
    rc = load_library().spconv_stage_timing(int(max_calls))
    if rc != SPCONV_OK:
        _raise(rc, "spconv_stage_timing")


def stage_times_ms() -> dict:
    """{stage: (summed ms, launches)} for the calls recorded since stage_timing(n)."""
    import numpy as np
    ms = np.zeros(len(STAGES), dtype=np.float64)
    cnt = np.zeros(len(STAGES), dtype=np.int64)
    n = load_library().spconv_stage_times_ms(ms.ctypes.data, cnt.ctypes.data, len(STAGES))
    if n < 0:
        _raise(SPCONV_ERR_CUDA, "spconv_stage_times_ms")
    return {STAGES[i]: (float(ms[i]), int(cnt[i])) for i in range(n)}
