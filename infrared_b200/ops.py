"""Tensor-level entry points over the C ABI (device memory and streams from PyTorch).

Every function takes CUDA tensors, checks shapes/dtypes/contiguity on the
host, and launches on ``torch.cuda.current_stream()`` without synchronising
or allocating anything but its outputs (which the caller may pass in), so
each one can run inside ``torch.cuda.graph`` capture. Device-side errors
(bad block ids, slots, metadata) are accumulated in a per-device int32 flag
word that :func:`check_device_errors` reads and clears.

There is no CPU path: CPU tensors raise ``ValueError``.
"""

from __future__ import annotations

import functools
import threading

import torch

from . import _lib
from ._lib import DEVERR_BITS, DecodeShape, check

_DTYPES = {
    torch.float32: _lib.IR_DTYPE_F32,
    torch.bfloat16: _lib.IR_DTYPE_BF16,
    torch.float16: _lib.IR_DTYPE_F16,
}


class DeviceError(RuntimeError):
    """Errors a kernel recorded on the device (see ``IR_DEVERR_*``)."""

    def __init__(self, bits: int):
        names = [n for b, n in DEVERR_BITS.items() if bits & b]
        super().__init__(f"infrared_b200 device error 0x{bits:x}: {', '.join(names)}")
        self.bits = bits


_state_lock = threading.Lock()
_err_flags: dict[int, torch.Tensor] = {}
_workspaces: dict[int, torch.Tensor] = {}


def _on_tensor_device(fn):
    """Run ``fn`` with its first tensor argument's device current.

    A kernel launch into a stream of a device other than the calling thread's
    current one fails, and callers such as infrared's engine run their loop
    in a worker thread whose current device is the process default (0);
    this switches to the tensors' device for the call when they differ."""

    @functools.wraps(fn)
    def wrapper(first, *args, **kwargs):
        idx = first.device.index if isinstance(first, torch.Tensor) and first.is_cuda else None
        if idx is not None and idx != torch.cuda.current_device():
            with torch.cuda.device(idx):
                return fn(first, *args, **kwargs)
        return fn(first, *args, **kwargs)

    return wrapper


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise _lib.UnsupportedShape(_lib.IR_ERR_UNSUPPORTED, f"dtype {dtype} not supported")


def _dev_index(t: torch.Tensor) -> int:
    if not t.is_cuda:
        raise ValueError("infrared_b200 kernels take CUDA tensors (no CPU path)")
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


def _index_of(device) -> int:
    if device is None:
        return torch.cuda.current_device()
    if isinstance(device, int):
        return device
    d = torch.device(device)
    return d.index if d.index is not None else torch.cuda.current_device()


def error_flag(device: torch.device | int | None = None) -> torch.Tensor:
    """The per-device int32 error word the kernels OR their error bits into."""
    idx = _index_of(device)
    t = _err_flags.get(idx)
    if t is not None:
        return t
    with _state_lock:
        t = _err_flags.get(idx)
        if t is None:
            t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
            _err_flags[idx] = t
    return t


def check_device_errors(device=None, clear: bool = True) -> None:
    """Synchronise on the flag word; raise :class:`DeviceError` if any bit is set."""
    flag = error_flag(device)
    bits = int(flag.item())
    if bits and clear:
        flag.zero_()
    if bits:
        raise DeviceError(bits)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device_index: int) -> int:
    return torch.cuda.current_stream(device_index).cuda_stream


# What a zeroed decode workspace turns on by default (ir_decode_shape.flags).
# Both features are opt-in (decode_workspace(dynamic=..., inline_merge=...)):
# on B200 the static shares with the separate merge kernel measured faster
# on every benchmark shape.
DYNAMIC_TAIL_DEFAULT = False
INLINE_MERGE_DEFAULT = False


def _default_flags(dynamic: bool | None = None, inline_merge: bool | None = None) -> int:
    dyn = DYNAMIC_TAIL_DEFAULT if dynamic is None else dynamic
    inl = INLINE_MERGE_DEFAULT if inline_merge is None else inline_merge
    return (_lib.IR_DECODE_DYNAMIC_TAIL if dyn else 0) | \
        (_lib.IR_DECODE_INLINE_MERGE if inl else 0)


def decode_workspace(nbytes: int, device, dynamic: bool | None = None,
                     inline_merge: bool | None = None) -> torch.Tensor:
    """A decode workspace of ``nbytes`` (at least 1 MiB) on ``device``, zero
    filled, marked with the features the decode calls given it may use:
    ``dynamic`` (``IR_DECODE_DYNAMIC_TAIL``: the last part of the tiles handed
    out as claimed units) and ``inline_merge`` (``IR_DECODE_INLINE_MERGE``:
    rows of at most 4 pieces merged in the decode kernel); None takes the
    module defaults. The kernels leave the header they count in zero after
    every call. Any other tensor given as a workspace gets neither."""
    t = torch.zeros(max(int(nbytes), 1 << 20), dtype=torch.uint8,
                    device=torch.device("cuda", _index_of(device)))
    # allocated inside a graph capture the zeroing only runs at replay: such
    # a workspace uses neither feature
    t._irb_flags = 0 if torch.cuda.is_current_stream_capturing() else \
        _default_flags(dynamic, inline_merge)
    return t


def _flags_of(ws: torch.Tensor | None) -> int:
    """Flags a call may ask for with this workspace (None: the cached one's)."""
    if ws is None:
        return _default_flags()
    return int(getattr(ws, "_irb_flags", 0))


def workspace(nbytes: int, device_index: int) -> torch.Tensor:
    """A cached, growing per-device workspace buffer (256-byte aligned, header
    zeroed: see :func:`decode_workspace`)."""
    t = _workspaces.get(device_index)
    if t is not None and t.numel() >= nbytes:
        return t
    with _state_lock:
        t = _workspaces.get(device_index)
        if t is None or t.numel() < nbytes:
            t = decode_workspace(nbytes, device_index)
            _workspaces[device_index] = t
    return t


def set_decode_path(path: int) -> None:
    """0 = automatic kernel choice, 1 = CUDA-core kernel, 2 = TMA kernel,
    3 = TMA kernel with one copy per (kv head, column half)."""
    check(_lib.load().ir_set_decode_path(path))
    _plans.clear()   # cached workspace sizes depend on the kernel choice


# --- pool scatter / gather ----------------------------------------------------


def _check_pool(pool: torch.Tensor, name: str) -> None:
    if pool.dim() != 3 or not pool.is_contiguous():
        raise ValueError(f"{name} must be a contiguous [num_slots, Hkv, D] tensor")


@_on_tensor_device
def cache_write(k: torch.Tensor, v: torch.Tensor, k_pool: torch.Tensor,
                v_pool: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """``k_pool[slot_mapping] = k; v_pool[slot_mapping] = v`` (one layer's pools)."""
    dev = _dev_index(k_pool)
    _check_pool(k_pool, "k_pool")
    _check_pool(v_pool, "v_pool")
    if k_pool.shape != v_pool.shape or k_pool.dtype != v_pool.dtype:
        raise ValueError("k_pool and v_pool differ")
    n = slot_mapping.numel()
    hkv, d = k_pool.shape[1], k_pool.shape[2]
    k = k.reshape(n, hkv, d)
    v = v.reshape(n, hkv, d)
    for t, nm in ((k, "k"), (v, "v")):
        if t.dtype != k_pool.dtype or t.device != k_pool.device:
            raise ValueError(f"{nm} must match the pool's dtype and device")
        if n and (t.stride(2) != 1 or t.stride(1) != d):
            raise ValueError(f"{nm} rows must be [Hkv, D] contiguous")
    slots = slot_mapping.reshape(-1)
    if slots.dtype != torch.int64 or not slots.is_contiguous() or slots.device != k_pool.device:
        raise ValueError("slot_mapping must be a contiguous int64 tensor on the pool's device")
    if n == 0:
        return
    lib = _lib.load()
    check(lib.ir_cache_write(
        k.data_ptr(), v.data_ptr(), k.stride(0), v.stride(0), k_pool.data_ptr(),
        v_pool.data_ptr(), slots.data_ptr(), n, hkv, d, k_pool.shape[0],
        dtype_code(k_pool.dtype), error_flag(dev).data_ptr(), _stream(dev)))


@_on_tensor_device
def cache_gather(pool: torch.Tensor, slots: torch.Tensor) -> torch.Tensor:
    """``pool[slots]`` for a 1-D or 2-D int64 slot tensor -> ``[*slots.shape, Hkv, D]``."""
    dev = _dev_index(pool)
    _check_pool(pool, "pool")
    flat = slots.reshape(-1)
    if flat.dtype != torch.int64 or flat.device != pool.device:
        raise ValueError("slots must be int64 on the pool's device")
    flat = flat.contiguous()
    out = torch.empty((flat.numel(), pool.shape[1], pool.shape[2]), dtype=pool.dtype,
                      device=pool.device)
    if flat.numel():
        check(_lib.load().ir_cache_gather(
            out.data_ptr(), pool.data_ptr(), flat.data_ptr(), flat.numel(), pool.shape[1],
            pool.shape[2], pool.shape[0], dtype_code(pool.dtype),
            error_flag(dev).data_ptr(), _stream(dev)))
    return out.reshape(*slots.shape, pool.shape[1], pool.shape[2])


@_on_tensor_device
def derive_block_metadata(gather_slots: torch.Tensor, mask: torch.Tensor, block_size: int,
                          block_tables: torch.Tensor | None = None,
                          context_lens: torch.Tensor | None = None):
    """``(gather_slots [B, T], decode mask [B, 1, 1, T]) -> (block_tables, context_lens)``.

    ``block_tables`` is int32 ``[B, ceil(T / block_size)]``, ``context_lens``
    int32 ``[B]``; both may be passed in (e.g. static graph buffers).
    """
    dev = _dev_index(gather_slots)
    if gather_slots.dim() != 2 or gather_slots.dtype != torch.int64:
        raise ValueError("gather_slots must be int64 [B, T]")
    b, t = gather_slots.shape
    if gather_slots.stride(1) != 1:
        gather_slots = gather_slots.contiguous()
    m2 = mask.reshape(b, t) if mask.numel() == b * t else None
    if m2 is None:
        raise ValueError("mask must have B*T elements ([B, 1, 1, T])")
    if m2.stride(1) != 1:
        m2 = m2.contiguous()
    nb = -(-t // block_size)
    if block_tables is None:
        block_tables = torch.empty((b, max(nb, 1)), dtype=torch.int32, device=gather_slots.device)
    if context_lens is None:
        context_lens = torch.empty((b,), dtype=torch.int32, device=gather_slots.device)
    if b:
        check(_lib.load().ir_derive_block_metadata(
            gather_slots.data_ptr(), gather_slots.stride(0), m2.data_ptr(), m2.stride(0),
            dtype_code(m2.dtype), b, t, block_size, block_tables.data_ptr(),
            block_tables.stride(0), context_lens.data_ptr(), error_flag(dev).data_ptr(),
            _stream(dev)))
    return block_tables, context_lens


# --- decode -------------------------------------------------------------------


def _shape(q: torch.Tensor, k_pool: torch.Tensor, block_tables: torch.Tensor,
           block_size: int, scale: float, out_stride: int,
           flags: int = 0) -> DecodeShape:
    b, h, d = q.shape
    hkv = k_pool.shape[1]
    s = DecodeShape()
    s.batch = b
    s.num_heads = h
    s.num_kv_heads = hkv
    s.head_dim = d
    s.block_size = block_size
    s.max_blocks = block_tables.shape[1]
    s.bt_stride = block_tables.stride(0) if block_tables.shape[0] else block_tables.shape[1]
    s.q_stride = q.stride(0)
    s.out_stride = out_stride
    s.num_slots = k_pool.shape[0]
    s.scale = float(scale)
    s.dtype = dtype_code(q.dtype)
    s.flags = flags
    return s


def _check_decode_inputs(q, k_pool, v_pool, block_tables, context_lens):
    _dev_index(q)
    if q.dim() != 3:
        raise ValueError("q must be [B, H, D]")
    if q.stride(2) != 1 or q.stride(1) != q.shape[2]:
        raise ValueError("q rows must be [H, D] contiguous")
    _check_pool(k_pool, "k_pool")
    _check_pool(v_pool, "v_pool")
    if k_pool.shape != v_pool.shape:
        raise ValueError("k_pool and v_pool shapes differ")
    if k_pool.dtype != q.dtype or v_pool.dtype != q.dtype:
        raise ValueError("q and the pools must share a dtype")
    if k_pool.shape[2] != q.shape[2]:
        raise ValueError("head_dim of q and pools differ")
    if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or \
            (block_tables.numel() and block_tables.stride(1) != 1):
        raise ValueError("block_tables must be int32 [B, max_blocks] with unit column stride")
    if context_lens.dtype != torch.int32 or not context_lens.is_contiguous():
        raise ValueError("context_lens must be contiguous int32 [B]")
    if block_tables.shape[0] != q.shape[0] or context_lens.numel() != q.shape[0]:
        raise ValueError("batch sizes of q, block_tables and context_lens differ")
    for t in (k_pool, v_pool, block_tables, context_lens):
        if t.device != q.device:
            raise ValueError("all tensors must be on the same device")


def decode_plan(q, k_pool, block_tables, block_size, scale=1.0, dynamic=False,
                inline_merge=None):
    """``(path, ctas_per_kv_head, workspace_bytes)`` the library picks for this
    call with a workspace from ``decode_workspace(dynamic=..., inline_merge=...)``
    (None: the module default)."""
    s = _shape(q, k_pool, block_tables, block_size, scale, q.shape[1] * q.shape[2],
               _default_flags(dynamic, inline_merge))
    lib = _lib.load()
    path, g = _lib.c_int(), _lib.c_int()
    check(lib.ir_paged_decode_plan(s, path, g))
    return path.value, g.value, lib.ir_paged_decode_workspace_size(s)


def _size_of(s: DecodeShape) -> int:
    lib = _lib.load()
    nbytes = lib.ir_paged_decode_workspace_size(s)
    if nbytes == 0:
        check(lib.ir_paged_decode_plan(s, None, None))
    return nbytes


def _ws_and_shape(make_shape, dev: int, ws: torch.Tensor | None, sized=None):
    """``(shape, workspace)`` of a decode call: the shape asks for the features
    the workspace is marked with (:func:`decode_workspace`; the cached
    per-device workspace has the module defaults unless it was allocated
    inside a graph capture). ``make_shape(flags)`` builds the shape;
    ``sized(flags)`` may return a cached ``(shape, bytes)``."""
    sized = sized or (lambda fl: (make_shape(fl), None))
    if ws is not None:
        s, nbytes = sized(_flags_of(ws))
        nbytes = _size_of(s) if nbytes is None else nbytes
        if ws.numel() < nbytes:
            raise ValueError(f"workspace of {ws.numel()} bytes < {nbytes} needed")
        return s, ws
    want = _flags_of(None)
    s, nbytes = sized(want)
    nbytes = _size_of(s) if nbytes is None else nbytes
    ws = workspace(nbytes, dev)
    got = _flags_of(ws)
    if got != want:   # fewer features need no more bytes
        s, _ = sized(got)
    return s, ws


# Validated call plans of paged_decode, keyed by everything the checks look
# at (shapes, strides, dtypes, devices, block size, scale): a repeated call
# (every layer of every decode step) skips the checks and the shape build.
_plans: dict = {}


def _decode_key(q, k_pool, v_pool, block_tables, context_lens, out, block_size, scale):
    return (q.shape, q.stride(), q.dtype, q.device, k_pool.shape, k_pool.stride(),
            k_pool.dtype, k_pool.device, v_pool.shape, v_pool.stride(), v_pool.dtype,
            v_pool.device, block_tables.shape, block_tables.stride(), block_tables.dtype,
            block_tables.device, context_lens.shape, context_lens.stride(),
            context_lens.dtype, context_lens.device, out.shape, out.stride(), out.dtype,
            block_size, float(scale))


@_on_tensor_device
def paged_decode(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                 block_tables: torch.Tensor, context_lens: torch.Tensor, scale: float,
                 block_size: int, out: torch.Tensor | None = None,
                 ws: torch.Tensor | None = None) -> torch.Tensor:
    """Decode attention: ``q [B, H, D]`` over paged K/V -> ``[B, H, D]`` (q's dtype).

    ``k_pool``/``v_pool`` are one layer's ``[num_slots, Hkv, D]`` pools,
    ``block_tables`` int32 ``[B, max_blocks]`` of block ids, ``context_lens``
    int32 ``[B]``. GQA: query head h reads kv head ``h // (H // Hkv)``.
    """
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    base = _decode_key(q, k_pool, v_pool, block_tables, context_lens, out, block_size, scale)

    def sized(flags):
        key = (base, flags)
        plan = _plans.get(key)
        if plan is None:
            _check_decode_inputs(q, k_pool, v_pool, block_tables, context_lens)
            if out.shape != q.shape or out.dtype != q.dtype or out.stride(2) != 1 or \
                    out.stride(1) != q.shape[2] or out.device != q.device:
                raise ValueError("out must be [B, H, D] with [H, D] contiguous rows")
            sh = _shape(q, k_pool, block_tables, block_size, scale, out.stride(0), flags)
            plan = (sh, _size_of(sh))
            if len(_plans) > 512:
                _plans.clear()
            _plans[key] = plan
        return plan

    dev = _dev_index(q)
    s, ws = _ws_and_shape(None, dev, ws, sized)
    check(_lib.load().ir_paged_decode(
        out.data_ptr(), q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(),
        block_tables.data_ptr(), context_lens.data_ptr(), s, ws.data_ptr(), ws.numel(),
        error_flag(dev).data_ptr(), _stream(dev)))
    return out


@_on_tensor_device
def paged_decode_write(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                       k_pool: torch.Tensor, v_pool: torch.Tensor,
                       slot_mapping: torch.Tensor, block_tables: torch.Tensor,
                       context_lens: torch.Tensor, scale: float, block_size: int,
                       out: torch.Tensor | None = None,
                       ws: torch.Tensor | None = None) -> torch.Tensor:
    """Cache write of ``k_new/v_new [B, Hkv, D]`` at ``slot_mapping`` fused with decode.

    ``slot_mapping[b]`` must be the slot of position ``context_lens[b] - 1``
    (the new token), as in the engine's decode step; otherwise the device
    error ``WRITE_SLOT`` is raised by :func:`check_device_errors`.
    """
    _check_decode_inputs(q, k_pool, v_pool, block_tables, context_lens)
    dev = _dev_index(q)
    b, hkv, d = q.shape[0], k_pool.shape[1], k_pool.shape[2]
    k_new = k_new.reshape(b, hkv, d)
    v_new = v_new.reshape(b, hkv, d)
    if k_new.stride(0) != v_new.stride(0) or k_new.stride(2) != 1 or k_new.stride(1) != d \
            or v_new.stride(2) != 1 or v_new.stride(1) != d:
        k_new, v_new = k_new.contiguous(), v_new.contiguous()
    if k_new.dtype != q.dtype or v_new.dtype != q.dtype:
        raise ValueError("k_new/v_new must match q's dtype")
    slots = slot_mapping.reshape(-1)
    if slots.dtype != torch.int64 or not slots.is_contiguous() or slots.numel() != b:
        raise ValueError("slot_mapping must be contiguous int64 [B]")
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    s, ws = _ws_and_shape(lambda fl: _shape(q, k_pool, block_tables, block_size, scale,
                                            out.stride(0), fl), dev, ws)
    check(_lib.load().ir_paged_decode_write(
        out.data_ptr(), q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(),
        k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0) if b else hkv * d,
        slots.data_ptr(), block_tables.data_ptr(), context_lens.data_ptr(), s,
        ws.data_ptr(), ws.numel(), error_flag(dev).data_ptr(), _stream(dev)))
    return out


@_on_tensor_device
def paged_decode_rope_write(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                            k_pool: torch.Tensor, v_pool: torch.Tensor,
                            slot_mapping: torch.Tensor, block_tables: torch.Tensor,
                            context_lens: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                            scale: float, block_size: int, out: torch.Tensor | None = None,
                            ws: torch.Tensor | None = None) -> torch.Tensor:
    """:func:`paged_decode_write` with RoPE applied in the kernel.

    ``q [B, H, D]`` and ``k_new [B, Hkv, D]`` are un-rotated (they may be
    row views of one QKV projection output); ``cos``/``sin`` are fp32
    ``[B, D]`` (or ``[B, 1, D]``) tables at the new token's position, as
    infrared's ``RotaryEmbedding`` returns them (layers.py:121-136). The pool
    and the output equal ``apply_rotary_pos_emb`` (layers.py:79-89) followed
    by :func:`paged_decode_write`, bit for bit.
    """
    _check_decode_inputs(q, k_pool, v_pool, block_tables, context_lens)
    dev = _dev_index(q)
    b, hkv, d = q.shape[0], k_pool.shape[1], k_pool.shape[2]
    k_new = k_new.reshape(b, hkv, d)
    v_new = v_new.reshape(b, hkv, d)
    if k_new.stride(0) != v_new.stride(0) or k_new.stride(2) != 1 or k_new.stride(1) != d \
            or v_new.stride(2) != 1 or v_new.stride(1) != d:
        k_new, v_new = k_new.contiguous(), v_new.contiguous()
    if k_new.dtype != q.dtype or v_new.dtype != q.dtype:
        raise ValueError("k_new/v_new must match q's dtype")
    cos = cos.reshape(b, d) if cos.dim() != 2 else cos
    sin = sin.reshape(b, d) if sin.dim() != 2 else sin
    for name, t in (("cos", cos), ("sin", sin)):
        if t.dtype != torch.float32 or t.device != q.device or t.shape != (b, d) \
                or t.stride(1) != 1:
            raise ValueError(f"{name} must be fp32 [B, D] rows on q's device")
    if cos.stride(0) != sin.stride(0):
        cos, sin = cos.contiguous(), sin.contiguous()
    slots = slot_mapping.reshape(-1)
    if slots.dtype != torch.int64 or not slots.is_contiguous() or slots.numel() != b:
        raise ValueError("slot_mapping must be contiguous int64 [B]")
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    s, ws = _ws_and_shape(lambda fl: _shape(q, k_pool, block_tables, block_size, scale,
                                            out.stride(0), fl), dev, ws)
    check(_lib.load().ir_paged_decode_rope_write(
        out.data_ptr(), q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(),
        k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0) if b else hkv * d,
        slots.data_ptr(), cos.data_ptr(), sin.data_ptr(), cos.stride(0) if b else d,
        block_tables.data_ptr(), context_lens.data_ptr(), s, ws.data_ptr(), ws.numel(),
        error_flag(dev).data_ptr(), _stream(dev)))
    return out


def _rope_rows(cos, sin, b, d, device):
    cos = cos.reshape(b, d) if cos.dim() != 2 else cos
    sin = sin.reshape(b, d) if sin.dim() != 2 else sin
    for name, t in (("cos", cos), ("sin", sin)):
        if t.dtype != torch.float32 or t.device != device or tuple(t.shape) != (b, d) \
                or t.stride(1) != 1:
            raise ValueError(f"{name} must be fp32 [B, D] rows on the tensors' device")
    if cos.stride(0) != sin.stride(0):
        cos, sin = cos.contiguous(), sin.contiguous()
    return cos, sin


@_on_tensor_device
def paged_decode_rope(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                      block_tables: torch.Tensor, context_lens: torch.Tensor,
                      cos: torch.Tensor, sin: torch.Tensor, scale: float, block_size: int,
                      out: torch.Tensor | None = None,
                      ws: torch.Tensor | None = None) -> torch.Tensor:
    """:func:`paged_decode` with RoPE applied to the un-rotated ``q`` in the
    kernel (``cos``/``sin`` fp32 ``[B, D]``): the step's K/V are already in the
    pool (:func:`kv_proj_rope_write`)."""
    _check_decode_inputs(q, k_pool, v_pool, block_tables, context_lens)
    dev = _dev_index(q)
    b, _, d = q.shape
    cos, sin = _rope_rows(cos, sin, b, d, q.device)
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    s, ws = _ws_and_shape(lambda fl: _shape(q, k_pool, block_tables, block_size, scale,
                                            out.stride(0), fl), dev, ws)
    check(_lib.load().ir_paged_decode_rope(
        out.data_ptr(), q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), cos.data_ptr(),
        sin.data_ptr(), cos.stride(0) if b else d, block_tables.data_ptr(),
        context_lens.data_ptr(), s, ws.data_ptr(), ws.numel(), error_flag(dev).data_ptr(),
        _stream(dev)))
    return out


@_on_tensor_device
def kv_proj_rope_write(x: torch.Tensor, w_k: torch.Tensor, w_v: torch.Tensor,
                       b_k: torch.Tensor | None, b_v: torch.Tensor | None,
                       cos: torch.Tensor | None, sin: torch.Tensor | None,
                       slot_mapping: torch.Tensor, k_pool: torch.Tensor,
                       v_pool: torch.Tensor) -> None:
    """``k_pool[slot] = rope(x @ w_k^T + b_k)``, ``v_pool[slot] = x @ w_v^T + b_v``
    for every row of ``x [N, hidden]`` in one tensor-core kernel
    (``ir_kv_proj_rope_write``): ``w_k`` / ``w_v`` are the ``nn.Linear``
    weights ``[Hkv * D, hidden]``, ``b_k`` / ``b_v`` their biases (or None),
    ``cos`` / ``sin`` fp32 ``[N, D]`` RoPE rows (or None: no RoPE), the pools
    one layer's ``[num_slots, Hkv, D]``; bf16 / fp16."""
    dev = _dev_index(x)
    _check_pool(k_pool, "k_pool")
    _check_pool(v_pool, "v_pool")
    if k_pool.shape != v_pool.shape or k_pool.dtype != v_pool.dtype:
        raise ValueError("k_pool and v_pool differ")
    hkv, d = k_pool.shape[1], k_pool.shape[2]
    x = x.reshape(-1, x.shape[-1])
    n, hidden = x.shape
    if x.stride(1) != 1:
        x = x.contiguous()
    for name, w in (("w_k", w_k), ("w_v", w_v)):
        if tuple(w.shape) != (hkv * d, hidden) or not w.is_contiguous():
            raise ValueError(f"{name} must be a contiguous [Hkv*D, hidden] weight")
    for name, t in (("x", x), ("w_k", w_k), ("w_v", w_v)):
        if t.dtype != k_pool.dtype or t.device != k_pool.device:
            raise ValueError(f"{name} must match the pool's dtype and device")
    for name, t in (("b_k", b_k), ("b_v", b_v)):
        if t is not None and (t.numel() != hkv * d or t.dtype != k_pool.dtype
                              or not t.is_contiguous() or t.device != k_pool.device):
            raise ValueError(f"{name} must be a contiguous [Hkv*D] bias of the pool's dtype")
    slots = slot_mapping.reshape(-1)
    if slots.dtype != torch.int64 or not slots.is_contiguous() or slots.numel() != n:
        raise ValueError("slot_mapping must be contiguous int64 [N]")
    rs = d
    if cos is not None:
        cos, sin = _rope_rows(cos, sin, n, d, x.device)
        rs = cos.stride(0) if n else d
    check(_lib.load().ir_kv_proj_rope_write(
        x.data_ptr(), x.stride(0) if n else hidden, n, hidden, w_k.data_ptr(), w_v.data_ptr(),
        _ptr(b_k), _ptr(b_v), _ptr(cos), _ptr(sin), rs, slots.data_ptr(), k_pool.data_ptr(),
        v_pool.data_ptr(), k_pool.shape[0], hkv, d, dtype_code(k_pool.dtype),
        error_flag(dev).data_ptr(), _stream(dev)))


@_on_tensor_device
def paged_decode_lse(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                     block_tables: torch.Tensor, context_lens: torch.Tensor, scale: float,
                     block_size: int, o: torch.Tensor | None = None,
                     lse: torch.Tensor | None = None, ws: torch.Tensor | None = None):
    """Partial decode: ``(o [B, H, D] fp32 normalised, lse [B, H] fp32 natural log)``."""
    _check_decode_inputs(q, k_pool, v_pool, block_tables, context_lens)
    dev = _dev_index(q)
    b, h, d = q.shape
    if o is None:
        o = torch.empty((b, h, d), dtype=torch.float32, device=q.device)
    if lse is None:
        lse = torch.empty((b, h), dtype=torch.float32, device=q.device)
    if not (o.is_contiguous() and lse.is_contiguous() and o.dtype == torch.float32
            and lse.dtype == torch.float32):
        raise ValueError("o and lse must be contiguous fp32")
    s, ws = _ws_and_shape(lambda fl: _shape(q, k_pool, block_tables, block_size, scale,
                                            h * d, fl), dev, ws)
    check(_lib.load().ir_paged_decode_lse(
        o.data_ptr(), lse.data_ptr(), q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(),
        block_tables.data_ptr(), context_lens.data_ptr(), s, ws.data_ptr(), ws.numel(),
        error_flag(dev).data_ptr(), _stream(dev)))
    return o, lse


@_on_tensor_device
def lse_merge(o_parts: torch.Tensor, lse_parts: torch.Tensor,
              dtype: torch.dtype = torch.float32,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """Combine ``o_parts [P, B, H, D]`` / ``lse_parts [P, B, H]`` (fp32) -> ``[B, H, D]``.

    Each part must be contiguous; the parts may sit at any stride (e.g. the
    rows of a packed all-gather buffer)."""
    dev = _dev_index(o_parts)
    if o_parts.dim() != 4 or lse_parts.shape != o_parts.shape[:3]:
        raise ValueError("o_parts must be [P, B, H, D] and lse_parts [P, B, H]")
    if o_parts.dtype != torch.float32 or lse_parts.dtype != torch.float32:
        raise ValueError("partials must be fp32")
    p, b, h, d = o_parts.shape
    if not (o_parts[0].is_contiguous() and lse_parts[0].is_contiguous()):
        o_parts, lse_parts = o_parts.contiguous(), lse_parts.contiguous()
    if out is None:
        out = torch.empty((b, h, d), dtype=dtype, device=o_parts.device)
    if out.stride(2) != 1 or out.stride(1) != d:
        raise ValueError("out rows must be [H, D] contiguous")
    check(_lib.load().ir_lse_merge(
        out.data_ptr(), out.stride(0), o_parts.data_ptr(), o_parts.stride(0),
        lse_parts.data_ptr(), lse_parts.stride(0), p, b, h, d, dtype_code(out.dtype),
        _stream(dev)))
    return out


# --- prefill / mixed varlen (Sq > 1) ----------------------------------------


def set_prefill_path(path: int) -> None:
    """0 auto, 1 rows as decode rows, 2 the tcgen05 tensor-core kernel, 3 its
    CTA-pair form (head_dim 128, cta_group::2; only on request)."""
    check(_lib.load().ir_set_prefill_path(int(path)))


def _prefill_shape(q, k_pool, block_tables, q_start, block_size, scale, out_stride):
    t, h, d = q.shape
    s = _lib.PrefillShape()
    s.num_seqs = q_start.numel() - 1
    s.total_q = t
    s.num_heads = h
    s.num_kv_heads = k_pool.shape[1]
    s.head_dim = d
    s.block_size = block_size
    s.max_blocks = block_tables.shape[1]
    s.bt_stride = block_tables.stride(0) if block_tables.shape[0] else block_tables.shape[1]
    s.q_stride = q.stride(0) if t else h * d
    s.out_stride = out_stride
    s.num_slots = k_pool.shape[0]
    s.scale = float(scale)
    s.dtype = dtype_code(q.dtype)
    return s


def prefill_plan(q, k_pool, block_tables, q_start, block_size, scale=1.0):
    """``(path, workspace_bytes)`` of :func:`paged_prefill` for these shapes."""
    s = _prefill_shape(q, k_pool, block_tables, q_start, block_size, scale,
                       q.shape[1] * q.shape[2])
    lib = _lib.load()
    path = _lib.c_int()
    check(lib.ir_paged_prefill_plan(s, path))
    return path.value, lib.ir_paged_prefill_workspace_size(s)


@_on_tensor_device
def paged_prefill(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                  block_tables: torch.Tensor, context_lens: torch.Tensor,
                  q_start: torch.Tensor, scale: float, block_size: int,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal paged attention of packed query rows ``q [total_q, H, D]``.

    Sequence ``s`` owns rows ``q_start[s] .. q_start[s+1]-1``, its last
    positions ``context_lens[s] - q_len .. context_lens[s] - 1`` (the pool
    already holds this step's K/V); each row attends its own sequence up to
    its position. ``block_tables`` int32 ``[S, max_blocks]``,
    ``context_lens`` int32 ``[S]``, ``q_start`` int32 ``[S + 1]``.
    """
    _dev_index(q)
    if q.dim() != 3 or q.stride(2) != 1 or q.stride(1) != q.shape[2]:
        raise ValueError("q must be [total_q, H, D] with [H, D] contiguous rows")
    _check_pool(k_pool, "k_pool")
    _check_pool(v_pool, "v_pool")
    if k_pool.shape != v_pool.shape or k_pool.dtype != q.dtype or v_pool.dtype != q.dtype:
        raise ValueError("pools must match each other and q's dtype")
    if k_pool.shape[2] != q.shape[2]:
        raise ValueError("head_dim of q and pools differ")
    for name, t, n in (("context_lens", context_lens, None), ("q_start", q_start, None)):
        if t.dtype != torch.int32 or not t.is_contiguous() or t.device != q.device:
            raise ValueError(f"{name} must be a contiguous int32 tensor on q's device")
    if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or \
            (block_tables.numel() and block_tables.stride(1) != 1) or \
            block_tables.device != q.device:
        raise ValueError("block_tables must be int32 [S, max_blocks] with unit column stride")
    nseq = q_start.numel() - 1
    if nseq < 0 or block_tables.shape[0] != nseq or context_lens.numel() != nseq:
        raise ValueError("q_start must have one more entry than block_tables / context_lens")
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    elif out.shape != q.shape or out.dtype != q.dtype or out.stride(2) != 1 or \
            out.stride(1) != q.shape[2]:
        raise ValueError("out must be [total_q, H, D] of q's dtype with contiguous rows")
    dev = _dev_index(q)
    s = _prefill_shape(q, k_pool, block_tables, q_start, block_size, scale,
                       out.stride(0) if out.shape[0] else q.shape[1] * q.shape[2])
    lib = _lib.load()
    nbytes = lib.ir_paged_prefill_workspace_size(s)
    ws = workspace(max(nbytes, 256), dev)
    check(lib.ir_paged_prefill(out.data_ptr(), q.data_ptr(), k_pool.data_ptr(),
                               v_pool.data_ptr(), block_tables.data_ptr(),
                               context_lens.data_ptr(), q_start.data_ptr(), s, ws.data_ptr(),
                               ws.numel(), error_flag(dev).data_ptr(), _stream(dev)))
    return out


@_on_tensor_device
def derive_varlen_metadata(gather_slots: torch.Tensor, mask: torch.Tensor, block_size: int):
    """``(block_tables [S, max_blocks], context_lens [S], q_start [S + 1])`` of
    one packed frame in infrared's form (``gather_slots [1, K]`` int64 and
    the additive ``mask [1, 1, Q, K]`` of inputs.py:38-94), built on the
    device; reading the sequence count back is one small synchronising copy.
    Inconsistent frames set device error bits (``check_device_errors``).
    """
    _dev_index(mask)
    gs = gather_slots.reshape(-1)
    if gs.dtype != torch.int64 or not gs.is_contiguous():
        gs = gs.to(torch.int64).contiguous()
    q, k = mask.shape[-2], mask.shape[-1]
    m2 = mask.reshape(q, k)
    if m2.stride(1) != 1:
        m2 = m2.contiguous()
    dev = _dev_index(mask)
    max_blocks = max(1, -(-k // block_size))
    bt = torch.empty((max(q, 1), max_blocks), dtype=torch.int32, device=mask.device)
    ctx = torch.empty(max(q, 1), dtype=torch.int32, device=mask.device)
    q_start = torch.empty(q + 1, dtype=torch.int32, device=mask.device)
    nseq = torch.empty(1, dtype=torch.int32, device=mask.device)
    scratch = torch.empty(max(3 * q, 1), dtype=torch.int32, device=mask.device)
    check(_lib.load().ir_derive_varlen_metadata(
        gs.data_ptr(), k, m2.data_ptr(), m2.stride(0) if q else k, dtype_code(m2.dtype), q,
        block_size, max_blocks, bt.data_ptr(), ctx.data_ptr(), q_start.data_ptr(),
        nseq.data_ptr(), scratch.data_ptr(), error_flag(dev).data_ptr(), _stream(dev)))
    s = int(nseq.item())
    return bt[:s], ctx[:s], q_start[:s + 1]
