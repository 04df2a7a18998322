"""Python binding of libmako_attn.so (include/mako_attn.h) over torch CUDA tensors.

The library is the product; this module only marshals torch tensors (device memory, the current stream) into the
C ABI.  It raises if the library is missing or a call fails -- there is no fallback of any kind.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmako_attn.so")

F16, BF16 = 0, 1
OK, EINVAL, ENOMEM, ECUDA, ENOTSUP = 0, -22, -12, -5, -95
OPT_PREFILL_KERNEL, OPT_DECODE_ROUTE, OPT_DECODE_CHUNK, OPT_KERNEL_TIMING, OPT_OUTPUT_16BIT, OPT_GRID_CTAS = 1, 2, 3, 4, 5, 6
UINT32_MAX = 0xFFFFFFFF

# Every symbol include/mako_attn.h declares, for the load check.
SYMBOLS = (
    "mako_attn_last_error", "mako_attn_version", "mako_attn_create", "mako_attn_destroy", "mako_attn_set_option",
    "mako_attn_launches", "mako_attn_device_error", "mako_attn_kernel_times", "mako_attention", "mako_attention_decode", "mako_cube_select", "mako_attention_sparse",
    "mako_attention_block_sparse", "mako_attention_decode_noalloc",
    "mako_peer_alloc", "mako_peer_free", "mako_peer_open", "mako_peer_close", "mako_group_create", "mako_group_connect",
    "mako_group_destroy", "mako_attention_gather", "mako_attention_decode_kv_sharded", "mako_group_connect_ptrs",
    "mako_group_area", "mako_heads", "mako_heads_norm", "mako_heads_partial", "mako_heads_clear",
    "mako_cube_layout", "mako_proj",
)


class CubeLayoutInfo(ctypes.Structure):
    """mako_cube_layout_info."""
    _fields_ = [(n, ctypes.c_uint32) for n in ("n_cubes", "rows", "q_pad", "k_pad", "dense0", "dense1", "topk",
                                               "stride")]
MAX_RANKS = 8


class IpcHandle(ctypes.Structure):
    """mako_ipc_handle: 64 opaque bytes a process passes to the others of its box."""
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]

_lib = None


class MakoError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{msg} (code {code})")
        self.code = code


def lib():
    """Loads libmako_attn.so and declares its signatures (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C mako-common_b200` (or __graft_entry__.build())")
    L = ctypes.CDLL(LIB_PATH)
    u32, i32, i64, p = ctypes.c_uint32, ctypes.c_int, ctypes.c_int64, ctypes.c_void_p
    L.mako_attn_last_error.restype = ctypes.c_char_p
    L.mako_attn_last_error.argtypes = []
    L.mako_attn_version.restype = i32
    L.mako_attn_create.argtypes = [i32, ctypes.POINTER(p)]
    L.mako_attn_destroy.argtypes = [p]
    L.mako_attn_set_option.argtypes = [p, i32, i64]
    L.mako_attn_launches.argtypes = [p, ctypes.POINTER(ctypes.c_uint64)]
    L.mako_attn_device_error.argtypes = [p, ctypes.POINTER(ctypes.c_int)]
    L.mako_attn_kernel_times.argtypes = [p, ctypes.POINTER(ctypes.c_float), u32, ctypes.POINTER(u32)]
    L.mako_attention.argtypes = [p, p, i32, p, p, p, p] + [u32] * 10
    L.mako_attention_decode.argtypes = [p, p, i32, p, p, p, p, u32, p, u32, u32, u32, u32, u32]
    L.mako_cube_select.argtypes = ([p, p, i32, p, p] + [u32] * 4 + [p, u32, ctypes.POINTER(p), ctypes.POINTER(p)]
                                   + [u32, u32])
    L.mako_attention_sparse.argtypes = [p, p, i32, p, p, p, p] + [u32] * 11 + [p, p, p, p]
    L.mako_attention_block_sparse.argtypes = [p, p, i32, p, p, p, p, u32, u32, u32, p, p, u32]
    L.mako_attention_decode_noalloc.argtypes = [p, i32, p, p, p, p, u32, p, u32, u32, u32, u32, u32]
    f32 = ctypes.c_float
    L.mako_heads.argtypes = [p, p, i32, p, u32, u32, u32, u32, u32, p, u32, p]
    L.mako_heads_norm.argtypes = [p, p, i32, p, u32, u32, u32, u32, u32, p, u32, p, f32, u32, p]
    L.mako_heads_partial.argtypes = [p, p, i32, p, u32, u32, u32, u32, u32, u32, u32, u32, p, p, f32, p, p]
    L.mako_heads_clear.argtypes = [p, p, i32, p, u32, u32, u32, u32]
    L.mako_proj.argtypes = [p, p, i32, p, p, p, u32, u32, u32, u32]
    L.mako_cube_layout.argtypes = [u32] * 6 + [ctypes.c_float, p, p, p, ctypes.POINTER(CubeLayoutInfo)]
    H = ctypes.POINTER(IpcHandle)
    L.mako_peer_alloc.argtypes = [p, ctypes.c_size_t, ctypes.POINTER(p), H]
    L.mako_peer_free.argtypes = [p, p]
    L.mako_peer_open.argtypes = [p, H, ctypes.POINTER(p)]
    L.mako_peer_close.argtypes = [p, p]
    L.mako_group_create.argtypes = [p, u32, u32, u32, ctypes.POINTER(p), H]
    L.mako_group_connect.argtypes = [p, H]
    L.mako_group_destroy.argtypes = [p]
    L.mako_group_connect_ptrs.argtypes = [p, ctypes.POINTER(p)]
    L.mako_group_area.argtypes = [p, ctypes.POINTER(p), ctypes.POINTER(ctypes.c_size_t)]
    L.mako_attention_gather.argtypes = [p, p, i32, p, p, p, ctypes.POINTER(p)] + [u32] * 10
    L.mako_attention_decode_kv_sharded.argtypes = [p, p, i32, p, p, p, p, u32, p, u32, u32, u32, u32, u32]
    for name in SYMBOLS:
        if name != "mako_attn_last_error":
            getattr(L, name).restype = i32
    _lib = L
    return L


def _check(rc: int):
    if rc != OK:
        raise MakoError(rc, lib().mako_attn_last_error().decode())


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    import torch
    s = torch.cuda.current_stream() if stream is None else stream
    return ctypes.c_void_p(s.cuda_stream)


def dtype_code(t) -> int:
    import torch
    if t.dtype == torch.float16:
        return F16
    if t.dtype == torch.bfloat16:
        return BF16
    raise TypeError(f"16-bit float tensors only, got {t.dtype}")


def attention_decode_noalloc(q, k, v, o, kv_len, max_kv_len, heads, kv_heads, dim, k_stride, stream=None):
    """mako_attention_decode_noalloc: the decode with its partials in the library's static device array -- no
    context, no device allocation (for callers that cannot allocate; calls must not overlap on the GPU)."""
    _check(lib().mako_attention_decode_noalloc(_stream(stream), dtype_code(q), _ptr(q), _ptr(k), _ptr(v), _ptr(o),
                                               kv_len.numel(), _ptr(kv_len), max_kv_len, heads, kv_heads, dim,
                                               k_stride))


class _DeviceArray:
    """A raw device allocation described by __cuda_array_interface__ (torch.as_tensor views it without a copy)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def device_view(ptr: int, shape, typestr: str = "<i2"):
    """A torch CUDA tensor over memory the library owns (e.g. cube_select's sel / nsel scratch)."""
    import torch
    return torch.as_tensor(_DeviceArray(ptr, shape, typestr), device="cuda")


class Context:
    """One mako_attn_ctx (its scratch and options) on a CUDA device."""

    def __init__(self, device: int = 0):
        self._h = ctypes.c_void_p()
        _check(lib().mako_attn_create(device, ctypes.byref(self._h)))
        self.device = device

    def close(self):
        if self._h:
            _check(lib().mako_attn_destroy(self._h))
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_option(self, option: int, value: int):
        _check(lib().mako_attn_set_option(self._h, option, value))

    def device_error(self) -> int:
        """Reads and clears the device error flag (0: every pipelined wait completed)."""
        n = ctypes.c_int()
        _check(lib().mako_attn_device_error(self._h, ctypes.byref(n)))
        return n.value

    def kernel_times(self, cap: int = 4096):
        """Milliseconds of each main kernel recorded while OPT_KERNEL_TIMING was on (waits for them; then forgets)."""
        buf = (ctypes.c_float * cap)()
        n = ctypes.c_uint32()
        _check(lib().mako_attn_kernel_times(self._h, buf, cap, ctypes.byref(n)))
        return [buf[i] for i in range(min(n.value, cap))]

    def launches(self) -> int:
        n = ctypes.c_uint64()
        _check(lib().mako_attn_launches(self._h, ctypes.byref(n)))
        return n.value

    # -- TransformerRuntime::attention (src/models/runtime.cpp:262-273)
    def attention(self, q, k, v, o, n_q, q_pad, n_k, k_pad, heads, kv_heads, q_pos0=0, block=UINT32_MAX, dim=128,
                  width=0, stream=None):
        _check(lib().mako_attention(self._h, _stream(stream), dtype_code(q), _ptr(q), _ptr(k), _ptr(v), _ptr(o), n_q,
                                    q_pad, n_k, k_pad, heads, kv_heads, q_pos0, block & UINT32_MAX, dim, width))

    def attention_decode(self, q, k, v, o, kv_len, max_kv_len, heads, kv_heads, dim, k_stride, stream=None):
        batch = kv_len.numel()
        _check(lib().mako_attention_decode(self._h, _stream(stream), dtype_code(q), _ptr(q), _ptr(k), _ptr(v), _ptr(o),
                                           batch, _ptr(kv_len), max_kv_len, heads, kv_heads, dim, k_stride))

    # -- TransformerRuntime::heads / heads_norm / heads_partial (src/models/runtime.cpp:215-260) and heads_clear;
    # y is a float16 or bfloat16 tensor [heads][n_pad][dim], x / cs / w float32 tensors (cs: (cos, sin) pairs)
    def proj(self, w, x, y, T, k, n, ldy=0, stream=None):
        """mako_proj: y[t][j] = sum_i x[t][i] w[j][i] (x [T][k], w [n][k] 16-bit of one type, y fp32 [T][ldy])."""
        _check(lib().mako_proj(self._h, _stream(stream), dtype_code(x), _ptr(w), _ptr(x), _ptr(y), T, k, n, ldy))

    def heads(self, x, ld, col0, heads, T, n_pad, cs, rope, y, stream=None):
        _check(lib().mako_heads(self._h, _stream(stream), dtype_code(y), _ptr(x), ld, col0, heads, T, n_pad, _ptr(cs),
                                rope, _ptr(y)))

    def heads_norm(self, x, ld, col0, heads, T, n_pad, cs, rope, w, eps, row0, y, stream=None):
        _check(lib().mako_heads_norm(self._h, _stream(stream), dtype_code(y), _ptr(x), ld, col0, heads, T, n_pad,
                                     _ptr(cs), rope, _ptr(w), eps, row0, _ptr(y)))

    def heads_partial(self, x, ld, col0, stride, dim, rot, heads, T, n_pad, cs, w, eps, y, map_=None, stream=None):
        _check(lib().mako_heads_partial(self._h, _stream(stream), dtype_code(y), _ptr(x), ld, col0, stride, dim, rot,
                                        heads, T, n_pad, _ptr(cs), _ptr(w), eps, _ptr(y), _ptr(map_)))

    def heads_clear(self, y, dim, n_pad, from_, heads, stream=None):
        _check(lib().mako_heads_clear(self._h, _stream(stream), dtype_code(y), _ptr(y), dim, n_pad, from_, heads))

    # -- TransformerRuntime::cube_select (src/models/runtime.cpp:286-303); returns (sel, nsel) as int16 tensor views
    # of the context's scratch ([heads][n_cubes][min(topk, n_cubes)] and [heads][n_cubes], uint16 bit patterns),
    # valid until the next cube_select on this context.
    def cube_select(self, q, k, heads, q_pad, k_pad, n_cubes, cnt, topk, local=0, stride=0, stream=None):
        sel, nsel = ctypes.c_void_p(), ctypes.c_void_p()
        _check(lib().mako_cube_select(self._h, _stream(stream), dtype_code(q), _ptr(q), _ptr(k), heads, q_pad, k_pad,
                                      n_cubes, _ptr(cnt), topk, ctypes.byref(sel), ctypes.byref(nsel), local, stride))
        kk = min(topk, n_cubes)
        return device_view(sel.value, (heads, n_cubes, kk)), device_view(nsel.value, (heads, n_cubes))

    # -- TransformerRuntime::attention_sparse (src/models/runtime.cpp:305-317); sel/nsel as tensors or raw pointers
    def attention_sparse(self, q, k, v, o, n_q, q_pad, n_k, k_pad, heads, kv_heads, width, n_cubes, topk, dense0,
                         dense1, sel, nsel, valid, map_, stream=None):
        sp = sel if isinstance(sel, int) or sel is None else sel.data_ptr()
        np_ = nsel if isinstance(nsel, int) or nsel is None else nsel.data_ptr()
        _check(lib().mako_attention_sparse(self._h, _stream(stream), dtype_code(q), _ptr(q), _ptr(k), _ptr(v), _ptr(o),
                                           n_q, q_pad, n_k, k_pad, heads, kv_heads, width, n_cubes, topk, dense0,
                                           dense1, ctypes.c_void_p(sp), ctypes.c_void_p(np_), _ptr(valid), _ptr(map_)))

    def attention_block_sparse(self, q, k, v, o, n, heads, kv_heads, lists, counts, stream=None):
        _check(lib().mako_attention_block_sparse(self._h, _stream(stream), dtype_code(q), _ptr(q), _ptr(k), _ptr(v),
                                                 _ptr(o), n, heads, kv_heads, _ptr(lists), _ptr(counts),
                                                 lists.shape[-1]))


# ---- multi-GPU (one process per GPU; handles travel through the caller's own channel) ------------------------------

def _handle_bytes(h: IpcHandle) -> bytes:
    return bytes(h.bytes)


def _handle_from(b: bytes) -> IpcHandle:
    h = IpcHandle()
    ctypes.memmove(h.bytes, b, 64)
    return h


class PeerBuffer:
    """A device buffer every rank maps (mako_peer_alloc here, mako_peer_open of the others' handles).

    `exchange(handle_bytes) -> list of every rank's handle bytes, in rank order` is the caller's channel, e.g.
    torch.distributed.all_gather_object.  `tensor` views this rank's buffer; `ptrs[r]` addresses rank r's."""

    def __init__(self, ctx: "Context", nbytes: int, rank: int, exchange, shape=None, typestr="<f4"):
        self._ctx = ctx
        self._ptr = ctypes.c_void_p()
        h = IpcHandle()
        _check(lib().mako_peer_alloc(ctx._h, nbytes, ctypes.byref(self._ptr), ctypes.byref(h)))
        handles = exchange(_handle_bytes(h))
        self.ptrs = []
        self._opened = []
        for r, hb in enumerate(handles):
            if r == rank:
                self.ptrs.append(self._ptr.value)
                continue
            q = ctypes.c_void_p()
            _check(lib().mako_peer_open(ctx._h, ctypes.byref(_handle_from(hb)), ctypes.byref(q)))
            self._opened.append(q)
            self.ptrs.append(q.value)
        itemsize = int(typestr[2:])
        self.tensor = device_view(self._ptr.value, shape or (nbytes // itemsize,), typestr)

    def close(self):
        for q in self._opened:
            lib().mako_peer_close(self._ctx._h, q)
        self._opened = []
        if self._ptr:
            lib().mako_peer_free(self._ctx._h, self._ptr)
            self._ptr = ctypes.c_void_p()


class Group:
    """This rank's mako_attn_group: created, its handle exchanged through `exchange`, connected."""

    def __init__(self, ctx: "Context", rank: int, n_ranks: int, max_rows: int, exchange=None):
        """exchange None: connect later with connect_ptrs (ranks sharing this process)."""
        self._ctx = ctx
        self._h = ctypes.c_void_p()
        h = IpcHandle()
        _check(lib().mako_group_create(ctx._h, rank, n_ranks, max_rows, ctypes.byref(self._h), ctypes.byref(h)))
        self.rank, self.n_ranks = rank, n_ranks
        if exchange is not None:
            handles = exchange(_handle_bytes(h))
            arr = (IpcHandle * n_ranks)(*[_handle_from(b) for b in handles])
            _check(lib().mako_group_connect(self._h, arr))

    def area(self):
        """(device pointer, bytes) of this rank's exchange area."""
        a, n = ctypes.c_void_p(), ctypes.c_size_t()
        _check(lib().mako_group_area(self._h, ctypes.byref(a), ctypes.byref(n)))
        return a.value, n.value

    def connect_ptrs(self, areas):
        arr = (ctypes.c_void_p * self.n_ranks)(*areas)
        _check(lib().mako_group_connect_ptrs(self._h, arr))

    def close(self):
        if self._h:
            _check(lib().mako_group_destroy(self._h))
            self._h = ctypes.c_void_p()

    def attention_gather(self, q, k, v, o_ptrs, n_q, q_pad, n_k, k_pad, heads, kv_heads, head0, width, q_pos0=0,
                         block=UINT32_MAX, stream=None):
        arr = (ctypes.c_void_p * len(o_ptrs))(*o_ptrs)
        _check(lib().mako_attention_gather(self._h, _stream(stream), dtype_code(q), _ptr(q), _ptr(k), _ptr(v), arr,
                                           n_q, q_pad, n_k, k_pad, heads, kv_heads, head0, q_pos0, block & UINT32_MAX,
                                           width))

    def attention_decode_kv_sharded(self, q, k, v, o, kv_len, max_kv_len, heads, kv_heads, dim, k_stride,
                                    stream=None):
        _check(lib().mako_attention_decode_kv_sharded(self._h, _stream(stream), dtype_code(q), _ptr(q), _ptr(k),
                                                      _ptr(v), _ptr(o), kv_len.numel(), _ptr(kv_len), max_kv_len,
                                                      heads, kv_heads, dim, k_stride))


def cube_layout(frames, ph, pw, rows_per_frame, video_row0, dense, keep):
    """mako_cube_layout: (map int32 [q_pad], valid uint8 [k_pad], cnt uint32 [n_cubes], info) as numpy arrays."""
    import numpy as np
    info = CubeLayoutInfo()
    L = lib()
    _check(L.mako_cube_layout(frames, ph, pw, rows_per_frame, video_row0, dense, keep, None, None, None,
                              ctypes.byref(info)))
    map_ = np.empty(info.q_pad, np.int32)
    valid = np.empty(info.k_pad, np.uint8)
    cnt = np.empty(max(info.n_cubes, 1), np.uint32)
    _check(L.mako_cube_layout(frames, ph, pw, rows_per_frame, video_row0, dense, keep,
                              map_.ctypes.data_as(ctypes.c_void_p), valid.ctypes.data_as(ctypes.c_void_p),
                              cnt.ctypes.data_as(ctypes.c_void_p), ctypes.byref(info)))
    return map_, valid, cnt[:info.n_cubes], info
