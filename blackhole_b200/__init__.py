"""blackhole_b200 -- B200 (sm_100a) NVFP4 x NVFP4 -> BF16 block-scaled GEMM.

Python mirror of the reference operator call ``blackhole::sm120::nvfp4_bf16_gemm``
(include/blackhole/sm120/nvfp4_gemm.hpp:588-637) over the C ABI in
include/blackhole_sm100.h.  Device memory may be passed as torch tensors (any dtype,
contiguous, on a CUDA device) or as raw integer device pointers.

There is no fallback: if libblackhole_sm100.so is missing or fails to load, every call
raises.
"""
from __future__ import annotations

import ctypes
import os

__all__ = [
    "LIB_PATH", "load", "nvfp4_bf16_gemm", "sf_storage_bytes", "sf_offset",
    "device_status", "BlackholeError", "nvfp4_quantize", "quantize_tensor",
    "nvfp4_bf16_gemm_ex", "workspace_bytes", "SCHEDULES", "nvfp4_bf16_gemm_noalloc",
    "selftest_bounded_wait", "mxfp4_bf16_gemm", "mxfp4_sf_storage_bytes", "mxfp4_quantize",
    "quantize_tensor_mxfp4", "mxf8f4_bf16_gemm", "mxfp8_quantize", "quantize_tensor_mxfp8",
    "nvfp4_bf16_gemm_gather", "peer_barrier", "ipc_get_handle", "ipc_open", "ipc_close",
    "selftest_skinny_partial_wait",
]

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libblackhole_sm100.so")

_lib = None


class BlackholeError(RuntimeError):
    """A C-ABI call returned a CUDA error code."""

    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} failed with cudaError {code} ({_CUDA_ERRORS.get(code, 'error')})")
        self.code = code


_CUDA_ERRORS = {0: "cudaSuccess", 1: "cudaErrorInvalidValue", 2: "cudaErrorMemoryAllocation",
                98: "cudaErrorInvalidDeviceFunction", 101: "cudaErrorInvalidDevice",
                209: "cudaErrorNoKernelImageForDevice", 400: "cudaErrorInvalidResourceHandle",
                700: "cudaErrorIllegalAddress", 801: "cudaErrorNotSupported"}


def load():
    """Load libblackhole_sm100.so (raises if it is absent: no fallback path exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing; build it with `python blackhole_b200/build.py`")
    L = ctypes.CDLL(LIB_PATH)
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    L.blackhole_sm100_nvfp4_bf16_gemm.restype = i32
    L.blackhole_sm100_nvfp4_bf16_gemm.argtypes = [i32, i32, i32, vp, vp, vp, vp, vp, ctypes.c_float, vp]
    L.blackhole_sm100_nvfp4_bf16_gemm_ex.restype = i32
    L.blackhole_sm100_nvfp4_bf16_gemm_ex.argtypes = [i32, i32, i32, vp, vp, vp, vp, vp, ctypes.c_float,
                                                     i32, vp, i64, vp]
    L.blackhole_sm100_nvfp4_bf16_gemm_noalloc.restype = i32
    L.blackhole_sm100_nvfp4_bf16_gemm_noalloc.argtypes = [i32, i32, i32, vp, vp, vp, vp, vp,
                                                          ctypes.c_float, vp]
    L.blackhole_sm100_mxfp4_bf16_gemm.restype = i32
    L.blackhole_sm100_mxfp4_bf16_gemm.argtypes = [i32, i32, i32, vp, vp, vp, vp, vp, ctypes.c_float, vp]
    L.blackhole_sm100_mxfp4_bf16_gemm_ex.restype = i32
    L.blackhole_sm100_mxfp4_bf16_gemm_ex.argtypes = [i32, i32, i32, vp, vp, vp, vp, vp, ctypes.c_float,
                                                     i32, vp, i64, vp]
    L.blackhole_sm100_mxf8f4_bf16_gemm.restype = i32
    L.blackhole_sm100_mxf8f4_bf16_gemm.argtypes = [i32, i32, i32, vp, vp, vp, vp, vp, ctypes.c_float, vp]
    L.blackhole_sm100_mxf8f4_bf16_gemm_ex.restype = i32
    L.blackhole_sm100_mxf8f4_bf16_gemm_ex.argtypes = [i32, i32, i32, vp, vp, vp, vp, vp,
                                                      ctypes.c_float, i32, vp, i64, vp]
    L.blackhole_sm100_mxfp8_quantize.restype = i32
    L.blackhole_sm100_mxfp8_quantize.argtypes = [vp, i32, i32, i32, vp, vp, vp]
    L.blackhole_sm100_mxfp4_sf_storage_bytes.restype = i64
    L.blackhole_sm100_mxfp4_sf_storage_bytes.argtypes = [i64, i64]
    L.blackhole_sm100_mxfp4_quantize.restype = i32
    L.blackhole_sm100_mxfp4_quantize.argtypes = [vp, i32, i32, i32, vp, vp, vp]
    L.blackhole_sm100_workspace_bytes.restype = i64
    L.blackhole_sm100_workspace_bytes.argtypes = [i32, i32, i32]
    L.blackhole_sm100_sf_storage_bytes.restype = i64
    L.blackhole_sm100_sf_storage_bytes.argtypes = [i64, i64]
    L.blackhole_sm100_sf_offset.restype = i64
    L.blackhole_sm100_sf_offset.argtypes = [i64, i64, i64]
    L.blackhole_sm100_device_status.restype = i32
    L.blackhole_sm100_device_status.argtypes = [i32, ctypes.POINTER(ctypes.c_uint), i32]
    L.blackhole_sm100_nvfp4_quantize.restype = i32
    L.blackhole_sm100_nvfp4_quantize.argtypes = [vp, i32, i32, i32, vp, vp, vp, vp]
    L.blackhole_sm100_selftest_skinny_partial_wait.restype = i32
    L.blackhole_sm100_selftest_skinny_partial_wait.argtypes = [i32, i32, i32, vp, vp, vp, vp, vp,
                                                               ctypes.c_float, vp, i64,
                                                               ctypes.c_uint64, vp]
    L.blackhole_sm100_selftest_bounded_wait.restype = i32
    L.blackhole_sm100_selftest_bounded_wait.argtypes = [ctypes.c_uint64, vp, vp]
    L.blackhole_sm100_nvfp4_bf16_gemm_gather.restype = i32
    L.blackhole_sm100_nvfp4_bf16_gemm_gather.argtypes = [i32, i32, i32, vp, vp, vp, vp, vp, i32, i64,
                                                         i64, ctypes.c_float, vp]
    L.blackhole_sm100_peer_barrier.restype = i32
    L.blackhole_sm100_peer_barrier.argtypes = [vp, i32, i32, ctypes.c_uint64, ctypes.c_uint64, vp]
    L.blackhole_sm100_ipc_get_handle.restype = i32
    L.blackhole_sm100_ipc_get_handle.argtypes = [vp, vp, ctypes.POINTER(ctypes.c_int64)]
    L.blackhole_sm100_ipc_open.restype = i32
    L.blackhole_sm100_ipc_open.argtypes = [vp, i64, ctypes.POINTER(ctypes.c_void_p)]
    L.blackhole_sm100_ipc_close.restype = i32
    L.blackhole_sm100_ipc_close.argtypes = [vp]
    L.blackhole_sm100_abi_version.restype = i32
    L.blackhole_sm100_abi_version.argtypes = []
    _lib = L
    return L


def _ptr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        if hasattr(x, "is_cuda") and not x.is_cuda:
            raise ValueError("tensor must live on a CUDA device")
        if hasattr(x, "is_contiguous") and not x.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return int(x.data_ptr())
    raise TypeError(f"cannot take a device pointer from {type(x)!r}")


def _stream(stream) -> int:
    if stream is None:
        try:
            import torch
            return int(torch.cuda.current_stream().cuda_stream)
        except Exception:
            return 0
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


def nvfp4_bf16_gemm(M: int, N: int, K: int, A, SFA, B, SFB, D, alpha: float = 1.0, stream=None) -> None:
    """D = bf16(alpha * A . B^T) for NVFP4 operands (asynchronous on `stream`).

    Same arguments as the reference call, in the same order, plus alpha:
    A (M x K/2 bytes, E2M1 packed, low nibble = even k), SFA (UE4M3, 128x4 layout,
    sf_storage_bytes(M, K) bytes), B (N x K/2), SFB, D (M x N bf16, row-major).
    Raises BlackholeError(cudaErrorInvalidValue) for unsupported shapes
    (M >= 1, N % 8 == 0, K % 32 == 0), null or misaligned pointers.
    """
    rc = load().blackhole_sm100_nvfp4_bf16_gemm(
        int(M), int(N), int(K), _ptr(A), _ptr(SFA), _ptr(B), _ptr(SFB), _ptr(D),
        float(alpha), _stream(stream))
    if rc != 0:
        raise BlackholeError("blackhole_sm100_nvfp4_bf16_gemm", rc)


SCHEDULES = {"auto": 0, "1sm": 1, "2sm": 2, "skinny": 3, "skinny_noprefetch": 4}


def nvfp4_bf16_gemm_ex(M: int, N: int, K: int, A, SFA, B, SFB, D, alpha: float = 1.0,
                       schedule: str = "auto", workspace=None, workspace_bytes: int = 0,
                       stream=None) -> None:
    """nvfp4_bf16_gemm with an explicit schedule ("auto", "1sm", "2sm", "skinny",
    "skinny_noprefetch": skinny without its early L2 prefetch, same results) and an
    optional caller-owned workspace for the skinny schedule (see workspace_bytes)."""
    if workspace is not None and hasattr(workspace, "numel") and not workspace_bytes:
        workspace_bytes = workspace.numel() * workspace.element_size()
    rc = load().blackhole_sm100_nvfp4_bf16_gemm_ex(
        int(M), int(N), int(K), _ptr(A), _ptr(SFA), _ptr(B), _ptr(SFB), _ptr(D), float(alpha),
        SCHEDULES[schedule], _ptr(workspace) if workspace is not None else None,
        int(workspace_bytes), _stream(stream))
    if rc != 0:
        raise BlackholeError("blackhole_sm100_nvfp4_bf16_gemm_ex", rc)


def mxfp4_bf16_gemm(M: int, N: int, K: int, A, SFA, B, SFB, D, alpha: float = 1.0, stream=None,
                    schedule: str = "auto", workspace=None, workspace_bytes: int = 0) -> None:
    """D = bf16(alpha * A . B^T) for MXFP4 operands (E2M1, one UE8M0 scale per 32 elements
    along K, 128x4 layout with 32-element groups: mxfp4_sf_storage_bytes(M|N, K) bytes).
    Same shapes, schedules and errors as nvfp4_bf16_gemm_ex."""
    if workspace is not None and hasattr(workspace, "numel") and not workspace_bytes:
        workspace_bytes = workspace.numel() * workspace.element_size()
    rc = load().blackhole_sm100_mxfp4_bf16_gemm_ex(
        int(M), int(N), int(K), _ptr(A), _ptr(SFA), _ptr(B), _ptr(SFB), _ptr(D), float(alpha),
        SCHEDULES[schedule], _ptr(workspace) if workspace is not None else None,
        int(workspace_bytes), _stream(stream))
    if rc != 0:
        raise BlackholeError("blackhole_sm100_mxfp4_bf16_gemm_ex", rc)


def mxf8f4_bf16_gemm(M: int, N: int, K: int, A, SFA, B, SFB, D, alpha: float = 1.0, stream=None,
                     schedule: str = "auto", workspace=None, workspace_bytes: int = 0) -> None:
    """D = bf16(alpha * A . B^T) with A MXFP8 (E4M3, one byte per element) and B MXFP4 (packed
    E2M1), UE8M0 scales per 32 along K on both (mxfp4_sf_storage_bytes(M|N, K) bytes each).
    K % 128 == 0; otherwise the shapes, schedules and errors of nvfp4_bf16_gemm_ex."""
    if workspace is not None and hasattr(workspace, "numel") and not workspace_bytes:
        workspace_bytes = workspace.numel() * workspace.element_size()
    rc = load().blackhole_sm100_mxf8f4_bf16_gemm_ex(
        int(M), int(N), int(K), _ptr(A), _ptr(SFA), _ptr(B), _ptr(SFB), _ptr(D), float(alpha),
        SCHEDULES[schedule], _ptr(workspace) if workspace is not None else None,
        int(workspace_bytes), _stream(stream))
    if rc != 0:
        raise BlackholeError("blackhole_sm100_mxf8f4_bf16_gemm_ex", rc)


def mxfp8_quantize(X, rows: int, K: int, q, sf, x_is_bf16: bool = False, stream=None) -> None:
    """Quantise X (rows x K, FP32 or BF16, K % 32 == 0) to MXFP8 (E4M3) on the GPU."""
    rc = load().blackhole_sm100_mxfp8_quantize(
        _ptr(X), 1 if x_is_bf16 else 0, int(rows), int(K), _ptr(q), _ptr(sf), _stream(stream))
    if rc != 0:
        raise BlackholeError("blackhole_sm100_mxfp8_quantize", rc)


def quantize_tensor_mxfp8(X, stream=None):
    """MXFP8 version of quantize_tensor: returns (q uint8 [rows, K], sf uint8)."""
    import torch

    if X.dim() != 2 or X.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("X must be a 2-D float32 or bfloat16 tensor")
    rows, K = X.shape
    q = torch.empty((rows, K), dtype=torch.uint8, device=X.device)
    sf = torch.empty(mxfp4_sf_storage_bytes(rows, K), dtype=torch.uint8, device=X.device)
    mxfp8_quantize(X, rows, K, q, sf, x_is_bf16=(X.dtype == torch.bfloat16), stream=stream)
    return q, sf


def mxfp4_sf_storage_bytes(mn: int, k: int) -> int:
    """Bytes of an (mn x k) MXFP4 scale-factor tensor (padding included)."""
    return int(load().blackhole_sm100_mxfp4_sf_storage_bytes(int(mn), int(k)))


def mxfp4_quantize(X, rows: int, K: int, packed, sf, x_is_bf16: bool = False, stream=None) -> None:
    """Quantise X (rows x K, FP32 or BF16, K % 32 == 0) to MXFP4 on the GPU (asynchronous)."""
    rc = load().blackhole_sm100_mxfp4_quantize(
        _ptr(X), 1 if x_is_bf16 else 0, int(rows), int(K), _ptr(packed), _ptr(sf), _stream(stream))
    if rc != 0:
        raise BlackholeError("blackhole_sm100_mxfp4_quantize", rc)


def quantize_tensor_mxfp4(X, stream=None):
    """MXFP4 version of quantize_tensor: returns (packed uint8 [rows, K/2], sf uint8)."""
    import torch

    if X.dim() != 2 or X.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("X must be a 2-D float32 or bfloat16 tensor")
    rows, K = X.shape
    packed = torch.empty((rows, K // 2), dtype=torch.uint8, device=X.device)
    sf = torch.empty(mxfp4_sf_storage_bytes(rows, K), dtype=torch.uint8, device=X.device)
    mxfp4_quantize(X, rows, K, packed, sf, x_is_bf16=(X.dtype == torch.bfloat16), stream=stream)
    return packed, sf


def nvfp4_bf16_gemm_gather(M: int, N: int, K: int, A, SFA, B, SFB, dst, col0: int, ldd: int,
                           alpha: float = 1.0, stream=None) -> None:
    """GEMM whose M x N result is written to columns [col0, col0 + N) of every buffer in
    `dst` (row-major BF16, rows `ldd` elements apart) from inside the kernel.  dst[0] must be
    this GPU's memory; the others may be other GPUs' buffers mapped with ipc_open.  The caller
    synchronises the ranks afterwards (nothing in the call waits for other GPUs)."""
    ptrs = dst if isinstance(dst, ctypes.Array) else pointer_array(dst)
    rc = load().blackhole_sm100_nvfp4_bf16_gemm_gather(
        int(M), int(N), int(K), _ptr(A), _ptr(SFA), _ptr(B), _ptr(SFB),
        ctypes.cast(ptrs, ctypes.c_void_p) if dst else None, len(dst), int(col0), int(ldd),
        float(alpha), _stream(stream))
    if rc != 0:
        raise BlackholeError("blackhole_sm100_nvfp4_bf16_gemm_gather", rc)


def pointer_array(bufs):
    """A ctypes array of the buffers' device pointers (build once, pass to every call)."""
    return (ctypes.c_void_p * max(1, len(bufs)))(*[_ptr(b) for b in bufs])


def peer_barrier(flags, world: int, rank: int, epoch: int, limit_ns: int = 1_000_000_000,
                 stream=None) -> None:
    """Stream-ordered barrier of a gathered N-split (see blackhole_sm100_peer_barrier):
    flags[q] is rank q's flag array as mapped here (a list, or a pointer_array)."""
    ptrs = flags if isinstance(flags, ctypes.Array) else pointer_array(flags)
    rc = load().blackhole_sm100_peer_barrier(ctypes.cast(ptrs, ctypes.c_void_p), int(world),
                                             int(rank), int(epoch), int(limit_ns), _stream(stream))
    if rc != 0:
        raise BlackholeError("blackhole_sm100_peer_barrier", rc)


def ipc_get_handle(buf):
    """(64-byte CUDA IPC handle of the allocation holding `buf`, byte offset of `buf` in it)."""
    h = (ctypes.c_char * 64)()
    off = ctypes.c_int64(0)
    rc = load().blackhole_sm100_ipc_get_handle(_ptr(buf), ctypes.cast(h, ctypes.c_void_p),
                                               ctypes.byref(off))
    if rc != 0:
        raise BlackholeError("blackhole_sm100_ipc_get_handle", rc)
    return bytes(h.raw), int(off.value)


def ipc_open(handle: bytes, offset: int) -> int:
    """Maps another process's buffer (from ipc_get_handle) on the current device; returns the
    device address of the same byte."""
    if len(handle) != 64:
        raise ValueError("an IPC handle is 64 bytes")
    h = (ctypes.c_char * 64).from_buffer_copy(handle)
    out = ctypes.c_void_p(0)
    rc = load().blackhole_sm100_ipc_open(ctypes.cast(h, ctypes.c_void_p), int(offset), ctypes.byref(out))
    if rc != 0:
        raise BlackholeError("blackhole_sm100_ipc_open", rc)
    return int(out.value)


def ipc_close(ptr: int) -> None:
    rc = load().blackhole_sm100_ipc_close(int(ptr))
    if rc != 0:
        raise BlackholeError("blackhole_sm100_ipc_close", rc)


def nvfp4_bf16_gemm_noalloc(M: int, N: int, K: int, A, SFA, B, SFB, D, alpha: float = 1.0,
                            stream=None) -> None:
    """The GEMM for M <= 16 without any device allocation, for callers that must not
    allocate at call time.  Its scratch lives in a fixed array inside the library (sized for
    M <= 16 on up to 160 SMs), shared by every call: calls that overlap on the GPU race.
    The first call on a device resolves the array's address; make it before any capture (a
    lookup that fails is tried again by the next call)."""
    rc = load().blackhole_sm100_nvfp4_bf16_gemm_noalloc(
        int(M), int(N), int(K), _ptr(A), _ptr(SFA), _ptr(B), _ptr(SFB), _ptr(D), float(alpha),
        _stream(stream))
    if rc != 0:
        raise BlackholeError("blackhole_sm100_nvfp4_bf16_gemm_noalloc", rc)


def selftest_skinny_partial_wait(M: int, N: int, K: int, A, SFA, B, SFB, D, alpha: float,
                                 workspace, partial_wait_ns: int, stream=None) -> None:
    """Test hook: the skinny schedule with the finishers' wait for partial sums bounded by
    partial_wait_ns (a tiny bound makes them give up, status bit 2).  workspace: a device
    buffer of at least workspace_bytes(M, N, K) bytes."""
    nbytes = int(workspace.numel() * workspace.element_size()) if hasattr(workspace, "numel") else 1 << 40
    rc = load().blackhole_sm100_selftest_skinny_partial_wait(
        int(M), int(N), int(K), _ptr(A), _ptr(SFA), _ptr(B), _ptr(SFB), _ptr(D), float(alpha),
        _ptr(workspace), nbytes, int(partial_wait_ns), _stream(stream))
    if rc != 0:
        raise BlackholeError("blackhole_sm100_selftest_skinny_partial_wait", rc)


def workspace_bytes(M: int, N: int, K: int) -> int:
    """Workspace bytes the skinny schedule needs on the current device (0 if unused)."""
    v = int(load().blackhole_sm100_workspace_bytes(int(M), int(N), int(K)))
    if v < 0:
        raise BlackholeError("blackhole_sm100_workspace_bytes", 1)
    return v


def sf_storage_bytes(mn: int, k: int) -> int:
    """Bytes of a (mn x k) scale-factor tensor in the 128x4 layout (padding included)."""
    return int(load().blackhole_sm100_sf_storage_bytes(int(mn), int(k)))


def sf_offset(mn: int, kg: int, k: int) -> int:
    return int(load().blackhole_sm100_sf_offset(int(mn), int(kg), int(k)))


def device_status(device: int = 0, clear: bool = True) -> int:
    """Status bits of this library's kernels on `device` (0 = no pipeline timed out).

    Synchronises the device."""
    out = ctypes.c_uint(0)
    rc = load().blackhole_sm100_device_status(int(device), ctypes.byref(out), 1 if clear else 0)
    if rc != 0:
        raise BlackholeError("blackhole_sm100_device_status", rc)
    return int(out.value)


def selftest_bounded_wait(limit_ns: int, result, stream=None) -> None:
    """Launches the bounded-wait self-test kernel (asynchronous): its producer warp times out
    after `limit_ns` and sets status bit 0; its consumer warp must leave through the CTA abort
    flag.  `result`: 4 device int64 words (completed flags of both warps, then their waits in
    ns)."""
    rc = load().blackhole_sm100_selftest_bounded_wait(int(limit_ns), _ptr(result), _stream(stream))
    if rc != 0:
        raise BlackholeError("blackhole_sm100_selftest_bounded_wait", rc)


def nvfp4_quantize(X, rows: int, K: int, packed, sf, scales, x_is_bf16: bool = False, stream=None) -> None:
    """Quantise X (rows x K, FP32 or BF16) to NVFP4 on the GPU (asynchronous).

    Writes packed E2M1 (rows*K/2 bytes), UE4M3 scale factors in the 128x4 layout
    (sf_storage_bytes(rows, K) bytes) and scales = [amax, g] (device float32[2])."""
    rc = load().blackhole_sm100_nvfp4_quantize(
        _ptr(X), 1 if x_is_bf16 else 0, int(rows), int(K), _ptr(packed), _ptr(sf), _ptr(scales),
        _stream(stream))
    if rc != 0:
        raise BlackholeError("blackhole_sm100_nvfp4_quantize", rc)


def quantize_tensor(X, stream=None):
    """Convenience wrapper for a 2-D torch tensor (float32 or bfloat16) on a CUDA device.

    Returns (packed uint8 [rows, K/2], sf uint8 [sf_storage_bytes], scales float32 [2])."""
    import torch

    if X.dim() != 2 or X.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("X must be a 2-D float32 or bfloat16 tensor")
    rows, K = X.shape
    packed = torch.empty((rows, K // 2), dtype=torch.uint8, device=X.device)
    sf = torch.empty(sf_storage_bytes(rows, K), dtype=torch.uint8, device=X.device)
    scales = torch.empty(2, dtype=torch.float32, device=X.device)
    nvfp4_quantize(X, rows, K, packed, sf, scales, x_is_bf16=(X.dtype == torch.bfloat16), stream=stream)
    return packed, sf, scales
