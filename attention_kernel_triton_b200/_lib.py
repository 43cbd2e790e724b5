"""ctypes binding of the C ABI in ``include/akt.h`` (``libakt.so``).

This is the only place Python touches native code.  The library is built
in-tree (``attention_kernel_triton_b200/libakt.so``); if it is missing, every
entry point raises ``RuntimeError`` -- there is no fallback path.
"""
from __future__ import annotations

import contextlib
import ctypes
import os
import threading
from ctypes import POINTER, Structure, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint, c_void_p

import torch  # loads the CUDA runtime the library links against

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libakt.so")

AKT_OK = 0
AKT_ERR_INVALID = 1
AKT_ERR_UNSUPPORTED = 2
AKT_ERR_CUDA = 3
AKT_ERR_WORKSPACE = 4
AKT_FLOAT16 = 0
AKT_BFLOAT16 = 1

DEVICE_STATUS_NAMES = {0: "ok", 1: "wait timeout", 2: "page id outside the pool",
                       3: "token index outside the sequence", 4: "malformed indptr",
                       5: "kept-index list longer than its buffer"}


class AktError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"akt error {code}: {msg}")
        self.code = code


class UnsupportedLayout(AktError):
    """The kernel cannot take this layout; the caller may retry with contiguous tensors."""


class DecodeDenseArgs(Structure):
    _fields_ = [
        ("q", c_void_p), ("q_stride_batch", c_int64), ("q_stride_head", c_int64), ("q_stride_dim", c_int64),
        ("k", c_void_p), ("k_stride_batch", c_int64), ("k_stride_head", c_int64), ("k_stride_token", c_int64),
        ("k_stride_dim", c_int64),
        ("v", c_void_p), ("v_stride_batch", c_int64), ("v_stride_head", c_int64), ("v_stride_token", c_int64),
        ("v_stride_dim", c_int64),
        ("out", c_void_p), ("out_stride_batch", c_int64), ("out_stride_head", c_int64), ("out_stride_dim", c_int64),
        ("batch", c_int32), ("num_qo_heads", c_int32), ("num_kv_heads", c_int32), ("seq_len", c_int32),
        ("head_dim", c_int32), ("dtype", c_int32), ("softmax_scale", c_float),
    ]


class DecodePagedArgs(Structure):
    _fields_ = [
        ("q", c_void_p), ("q_stride_batch", c_int64), ("q_stride_head", c_int64), ("q_stride_dim", c_int64),
        ("kv_cache", c_void_p), ("kv_stride_page", c_int64), ("kv_stride_kv", c_int64), ("kv_stride_head", c_int64),
        ("kv_stride_token", c_int64), ("kv_stride_dim", c_int64), ("num_pages", c_int64),
        ("kv_page_indptr", c_void_p), ("kv_page_indices", c_void_p), ("kv_last_page_len", c_void_p),
        ("num_page_entries", c_int64),
        ("out", c_void_p), ("out_stride_batch", c_int64), ("out_stride_head", c_int64), ("out_stride_dim", c_int64),
        ("batch", c_int32), ("num_qo_heads", c_int32), ("num_kv_heads", c_int32), ("page_size", c_int32),
        ("head_dim", c_int32), ("dtype", c_int32), ("softmax_scale", c_float),
    ]


class SparseDenseArgs(Structure):
    _fields_ = [
        ("q", c_void_p), ("q_stride_batch", c_int64), ("q_stride_head", c_int64), ("q_stride_dim", c_int64),
        ("k", c_void_p), ("k_stride_batch", c_int64), ("k_stride_head", c_int64), ("k_stride_token", c_int64),
        ("k_stride_dim", c_int64),
        ("v", c_void_p), ("v_stride_batch", c_int64), ("v_stride_head", c_int64), ("v_stride_token", c_int64),
        ("v_stride_dim", c_int64),
        ("sparse_ind", c_void_p), ("ind_stride_batch", c_int64), ("ind_stride_head", c_int64),
        ("ind_stride_pos", c_int64),
        ("sparse_nnz", c_void_p), ("nnz_stride_batch", c_int64), ("nnz_stride_head", c_int64),
        ("out", c_void_p), ("out_stride_batch", c_int64), ("out_stride_head", c_int64), ("out_stride_dim", c_int64),
        ("batch", c_int32), ("num_qo_heads", c_int32), ("num_kv_heads", c_int32), ("seq_len", c_int32),
        ("head_dim", c_int32), ("max_nnz", c_int32), ("dtype", c_int32), ("softmax_scale", c_float),
    ]


class SparsePagedArgs(Structure):
    _fields_ = [
        ("q", c_void_p), ("q_stride_batch", c_int64), ("q_stride_head", c_int64), ("q_stride_dim", c_int64),
        ("kv_cache", c_void_p), ("kv_stride_page", c_int64), ("kv_stride_kv", c_int64), ("kv_stride_head", c_int64),
        ("kv_stride_token", c_int64), ("kv_stride_dim", c_int64), ("num_pages", c_int64),
        ("kv_page_indptr", c_void_p), ("kv_page_indices", c_void_p), ("num_page_entries", c_int64),
        ("sparse_ind", c_void_p), ("ind_stride_batch", c_int64), ("ind_stride_head", c_int64),
        ("ind_stride_pos", c_int64),
        ("sparse_nnz", c_void_p), ("nnz_stride_batch", c_int64), ("nnz_stride_head", c_int64),
        ("magicpig_k", c_void_p), ("magicpig_l", c_void_p), ("param_stride_batch", c_int64),
        ("param_stride_head", c_int64),
        ("out", c_void_p), ("out_stride_batch", c_int64), ("out_stride_head", c_int64), ("out_stride_dim", c_int64),
        ("batch", c_int32), ("num_qo_heads", c_int32), ("num_kv_heads", c_int32), ("page_size", c_int32),
        ("head_dim", c_int32), ("max_nnz", c_int32), ("dtype", c_int32), ("softmax_scale", c_float),
    ]


class PrefillArgs(Structure):
    _fields_ = [
        ("q", c_void_p), ("q_stride_batch", c_int64), ("q_stride_head", c_int64), ("q_stride_token", c_int64),
        ("q_stride_dim", c_int64),
        ("k", c_void_p), ("k_stride_batch", c_int64), ("k_stride_head", c_int64), ("k_stride_token", c_int64),
        ("k_stride_dim", c_int64),
        ("v", c_void_p), ("v_stride_batch", c_int64), ("v_stride_head", c_int64), ("v_stride_token", c_int64),
        ("v_stride_dim", c_int64),
        ("out", c_void_p), ("out_stride_batch", c_int64), ("out_stride_head", c_int64),
        ("out_stride_token", c_int64), ("out_stride_dim", c_int64),
        ("varlen", c_void_p),
        ("batch", c_int32), ("num_qo_heads", c_int32), ("num_kv_heads", c_int32), ("seq_len", c_int32),
        ("head_dim", c_int32), ("causal", c_int32), ("dtype", c_int32), ("softmax_scale", c_float),
    ]


class MaskToIndexArgs(Structure):
    _fields_ = [
        ("mask", c_void_p), ("mask_stride_batch", c_int64), ("mask_stride_head", c_int64),
        ("sparse_ind", c_void_p), ("ind_stride_batch", c_int64), ("ind_stride_head", c_int64),
        ("sparse_nnz", c_void_p), ("nnz_stride_batch", c_int64), ("nnz_stride_head", c_int64),
        ("batch", c_int32), ("num_heads", c_int32), ("seq_len", c_int32), ("max_kept", c_int32),
        ("keep_first_if_empty", c_int32),
    ]


class IndexToMaskArgs(Structure):
    _fields_ = [
        ("sparse_ind", c_void_p), ("ind_stride_batch", c_int64), ("ind_stride_head", c_int64),
        ("sparse_nnz", c_void_p), ("nnz_stride_batch", c_int64), ("nnz_stride_head", c_int64),
        ("mask", c_void_p), ("mask_stride_batch", c_int64), ("mask_stride_head", c_int64),
        ("batch", c_int32), ("num_heads", c_int32), ("seq_len", c_int32), ("max_kept", c_int32),
    ]


class AppendPagedArgs(Structure):
    _fields_ = [
        ("kv_cache", c_void_p), ("kv_stride_page", c_int64), ("kv_stride_kv", c_int64), ("kv_stride_head", c_int64),
        ("kv_stride_token", c_int64), ("kv_stride_dim", c_int64), ("num_pages", c_int64),
        ("kv_page_indptr", c_void_p), ("kv_page_indices", c_void_p), ("kv_last_page_len", c_void_p),
        ("num_page_entries", c_int64),
        ("append_k", c_void_p), ("k_stride_token", c_int64), ("k_stride_head", c_int64), ("k_stride_dim", c_int64),
        ("append_v", c_void_p), ("v_stride_token", c_int64), ("v_stride_head", c_int64), ("v_stride_dim", c_int64),
        ("append_indptr", c_void_p), ("num_append", c_int64),
        ("batch", c_int32), ("num_kv_heads", c_int32), ("page_size", c_int32), ("head_dim", c_int32),
        ("dtype", c_int32),
    ]


AKT_MAX_PEERS = 8


class PeerExchange(Structure):
    _fields_ = [
        ("peer_data", c_void_p * AKT_MAX_PEERS), ("peer_flags", c_void_p * AKT_MAX_PEERS), ("counter", c_void_p),
        ("merge_counter", c_void_p), ("world", c_int32), ("rank", c_int32), ("epoch", ctypes.c_uint32),
    ]


# name -> (restype, argtypes); every function declared in include/akt.h
SIGNATURES = {
    "akt_abi_version": (c_int, []),
    "akt_last_error": (c_char_p, []),
    "akt_device_status": (c_int, [c_int, POINTER(c_uint)]),
    "akt_clear_device_status": (c_int, [c_int]),
    "akt_profile_enable": (c_int, [c_int]),
    "akt_profile_read": (c_int, [POINTER(ctypes.c_double), POINTER(c_int64)]),
    "akt_prefill": (c_int, [POINTER(PrefillArgs), c_void_p]),
    "akt_prefill_with_lse": (c_int, [POINTER(PrefillArgs), c_void_p, c_int64, c_int64, c_void_p]),
    "akt_decode_dense_workspace_size": (c_size_t, [POINTER(DecodeDenseArgs)]),
    "akt_decode_dense": (c_int, [POINTER(DecodeDenseArgs), c_void_p, c_size_t, c_void_p]),
    "akt_decode_paged_workspace_size": (c_size_t, [POINTER(DecodePagedArgs)]),
    "akt_decode_paged": (c_int, [POINTER(DecodePagedArgs), c_void_p, c_size_t, c_void_p]),
    "akt_decode_paged_noalloc": (c_int, [POINTER(DecodePagedArgs), c_void_p]),
    "akt_sparse_dense_workspace_size": (c_size_t, [POINTER(SparseDenseArgs)]),
    "akt_sparse_dense": (c_int, [POINTER(SparseDenseArgs), c_void_p, c_size_t, c_void_p]),
    "akt_sparse_paged_workspace_size": (c_size_t, [POINTER(SparsePagedArgs)]),
    "akt_sparse_paged": (c_int, [POINTER(SparsePagedArgs), c_void_p, c_size_t, c_void_p]),
    "akt_magicpig_paged_workspace_size": (c_size_t, [POINTER(SparsePagedArgs)]),
    "akt_magicpig_paged": (c_int, [POINTER(SparsePagedArgs), c_void_p, c_size_t, c_void_p]),
    "akt_sparse_dense_partial": (c_int, [POINTER(SparseDenseArgs), c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "akt_sparse_paged_partial": (c_int, [POINTER(SparsePagedArgs), c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "akt_magicpig_paged_partial": (c_int, [POINTER(SparsePagedArgs), c_void_p, c_void_p, c_void_p, c_size_t,
                                           c_void_p]),
    "akt_lse_merge": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int32, c_int64, c_int32, c_void_p, c_int64,
                              c_int32, c_void_p]),
    "akt_sparse_dense_csr": (c_int, [POINTER(SparseDenseArgs), c_void_p, c_int64, c_void_p, c_size_t, c_void_p]),
    "akt_sparse_paged_csr": (c_int, [POINTER(SparsePagedArgs), c_void_p, c_int64, c_void_p, c_size_t, c_void_p]),
    "akt_magicpig_paged_csr": (c_int, [POINTER(SparsePagedArgs), c_void_p, c_int64, c_void_p, c_size_t,
                                       c_void_p]),
    "akt_append_paged_kv": (c_int, [POINTER(AppendPagedArgs), c_void_p]),
    "akt_ipc_alloc": (c_int, [c_size_t, POINTER(c_void_p), c_void_p]),
    "akt_ipc_open": (c_int, [c_void_p, POINTER(c_void_p)]),
    "akt_ipc_close": (c_int, [c_void_p]),
    "akt_ipc_free": (c_int, [c_void_p]),
    "akt_sparse_dense_partial_peer": (c_int, [POINTER(SparseDenseArgs), POINTER(PeerExchange), c_void_p, c_size_t,
                                              c_void_p]),
    "akt_lse_merge_peer": (c_int, [POINTER(PeerExchange), c_int64, c_int32, c_void_p, c_int64, c_int32, c_void_p]),
    "akt_sparse_dense_split_peer": (c_int, [POINTER(SparseDenseArgs), POINTER(PeerExchange), c_void_p, c_size_t,
                                            c_void_p]),
    "akt_mask_to_sparse_index": (c_int, [POINTER(MaskToIndexArgs), c_void_p]),
    "akt_sparse_index_to_mask": (c_int, [POINTER(IndexToMaskArgs), c_void_p]),
}

_lib = None
_lock = threading.Lock()


def lib():
    """Load ``libakt.so`` once; raise if it is absent (no fallback)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python -m attention_kernel_triton_b200.build`")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                if L.akt_abi_version() != 1:
                    raise RuntimeError("libakt.so ABI version mismatch")
                _lib = L
    return _lib


def check(rc: int) -> None:
    if rc == AKT_OK:
        return
    msg = (lib().akt_last_error() or b"").decode(errors="replace")
    if rc == AKT_ERR_UNSUPPORTED:
        raise UnsupportedLayout(rc, msg)
    raise AktError(rc, msg)


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float16:
        return AKT_FLOAT16
    if t.dtype == torch.bfloat16:
        return AKT_BFLOAT16
    raise TypeError(f"unsupported dtype {t.dtype}: float16 or bfloat16 expected")


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device) -> int:
    """torch's current stream on ``device`` as a ``cudaStream_t`` value (the raw
    query when torch has it: it skips building a Stream object per call)."""
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def on_device(device: torch.device):
    """Context that makes ``device`` current for the launches inside it; no
    device switch (and no context-manager cost) when it already is."""
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """Scratch from torch's caching allocator (no cudaMalloc per call)."""
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def device_status(device: int = 0, clear: bool = False) -> int:
    v = c_uint(0)
    check(lib().akt_device_status(int(device), ctypes.byref(v)))
    if clear:
        check(lib().akt_clear_device_status(int(device)))
    return int(v.value)


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if not t.is_cuda:
            raise ValueError("all tensors must be CUDA tensors (this library has no CPU path)")
        if t.device != dev:
            raise ValueError("all tensors must be on the same device")
    return dev


class profile_kernels:
    """Context manager: time the main kernel of every entry point called inside.

    ``with profile_kernels() as p: ...`` then ``p.total_ms`` / ``p.launches``."""

    def __enter__(self):
        check(lib().akt_profile_enable(1))
        self.total_ms, self.launches = 0.0, 0
        return self

    def __exit__(self, *exc):
        ms = ctypes.c_double(0)
        n = c_int64(0)
        check(lib().akt_profile_read(ctypes.byref(ms), ctypes.byref(n)))
        check(lib().akt_profile_enable(0))
        self.total_ms, self.launches = float(ms.value), int(n.value)
        return False


def index_strides(sparse_ind: torch.Tensor, sparse_nnz: torch.Tensor):
    """(ind batch, head, pos) and (nnz batch, head) element strides; nnz may be [B,H] or [B,H,1]."""
    if sparse_ind.dim() != 3:
        raise ValueError("sparse_ind must be [B, Hq, L_max]")
    if sparse_nnz.dim() not in (2, 3) or (sparse_nnz.dim() == 3 and sparse_nnz.shape[2] != 1):
        raise ValueError("sparse_nnz must be [B, Hq] or [B, Hq, 1]")
    return sparse_ind.stride(), (sparse_nnz.stride(0), sparse_nnz.stride(1))


def as_int32(t: torch.Tensor, device) -> torch.Tensor:
    if t.dtype != torch.int32 or t.device != device:
        t = t.to(device=device, dtype=torch.int32)
    return t


def run_with_layout_retry(call, make_contiguous):
    """Call the entry point; if it rejects the layout, retry once on contiguous copies."""
    rc = call()
    if rc == AKT_ERR_UNSUPPORTED:
        make_contiguous()
        rc = call()
    check(rc)
