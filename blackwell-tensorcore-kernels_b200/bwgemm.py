"""Python face of libbwgemm.so (the C ABI declared in include/bwgemm.h).

Used by bench.py, tests/ and __graft_entry__. Device memory and streams come from torch;
every call goes through the C ABI with raw pointers, so what runs is the in-tree CUDA
library. There is no fallback: if the shared library is missing or fails to load, every
entry point raises.

Reference interface mirrored (paths within waynehacking8/blackwell-tensorcore-kernels):
  launch_<name>(A, B, C, M, N, K)  src/main.cu:18-39 -> launch(name, A, B, C) below, with the
  same staging semantics (FP32 inputs are cast/quantised by the launcher, cached by pointer
  identity and shape, src/gemm_mma.cu:152-168, src/gemm_mma_fp8.cu:230-264).
"""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

_HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(_HERE)
LIB_PATH = os.path.join(_HERE, "libbwgemm.so")
HEADER = os.path.join(REPO, "include", "bwgemm.h")

BW_OK, BW_ERR_INVALID, BW_ERR_CUDA, BW_ERR_TIMEOUT, BW_ERR_UNSUPPORTED = 0, 1, 2, 3, 4
OUT_F32, OUT_BF16 = 0, 1
SCALE_NONE, SCALE_FIXED8, SCALE_AMAX = 0, 1, 2
FP4_PACKED, FP4_BYTE_SHL2 = 0, 1
MX_UNIT_FIXED8, MX_BLOCK32 = 0, 1
DTYPE_F16, DTYPE_FP8, DTYPE_FP4, DTYPE_MXFP4 = 0, 1, 2, 3


class Shard(ctypes.Structure):
    """bw_shard_t: one GPU's part of a single-process sharded GEMM (include/bwgemm.h)."""

    _fields_ = [("device", ctypes.c_int), ("A", ctypes.c_void_p), ("B", ctypes.c_void_p),
                ("sfA", ctypes.c_void_p), ("sfB", ctypes.c_void_p), ("scale_a", ctypes.c_void_p),
                ("scale_b", ctypes.c_void_p), ("C", ctypes.c_void_p), ("C_gathered", ctypes.c_void_p),
                ("stream", ctypes.c_void_p)]


class BwError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"bwgemm error {code}: {msg}")
        self.code = code


_lib = None


def build(tools: bool = False) -> None:
    """Compile the library (and optionally gemm_bench / tc_rate_probe) for sm_100a in-tree."""
    targets = ["all"] + (["tools"] if tools else [])
    subprocess.run(["make", "-s", "-C", _HERE, *targets], check=True)


def declared_functions() -> list[str]:
    """Names of the entry points include/bwgemm.h declares."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^\s*(?:int|size_t|const char\*)\s+(bw_\w+)\s*\(", text, flags=re.M)


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: run __graft_entry__.build() (make -C {_HERE})")
    L = ctypes.CDLL(LIB_PATH)
    P, I, LL = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
    sig = {
        "bw_init": [I],
        "bw_shutdown": [],
        "bw_version": [],
        "bw_num_sms": [I],
        "bw_device_state_ready": [I],
        "bw_device_status": [P, P],
        "bw_set_wait_budget_ns": [ctypes.c_ulonglong],
        "bw_set_trace_buffer": [P, I],
        "bw_selftest_bounded_wait": [ctypes.c_ulonglong, P],
        "bw_gemm_f16": [P, P, P, I, I, I, P],
        "bw_gemm_f16_bt": [P, P, P, I, I, I, P],
        "bw_gemm_fp8": [P, P, P, P, P, I, I, I, I, P],
        "bw_gemm_mxfp4": [P, P, P, P, P, P, P, I, I, I, I, P],
        "bw_gemm_fp4": [P, P, P, P, P, I, I, I, I, P],
        "bw_quantize_f16": [P, P, LL, P],
        "bw_quantize_fp8": [P, P, P, I, I, I, I, P],
        "bw_quantize_fp8_noalloc": [P, P, P, I, I, I, I, P],
        "bw_quantize_fp4": [P, P, P, I, I, I, I, I, P],
        "bw_quantize_mxfp4": [P, P, P, I, I, I, I, P],
        "bw_unshard_columns": [P, P, I, I, I, P],
        "bw_unshard_columns_bf16": [P, P, I, I, I, P],
        "bw_gemm_sharded": [I, I, P, I, I, I, I, I],
        "bw_gemm_f16_allgather": [P, P, P, P, I, I, I, I, I, P],
        "bw_gemm_fp8_allgather": [P, P, P, P, P, I, P, I, I, I, I, I, P],
        "bw_gemm_f16_allgather_multicast": [P, P, P, I, I, I, I, I, P],
        "bw_gemm_fp8_allgather_multicast": [P, P, P, P, P, I, I, I, I, I, I, P],
        "bw_ipc_malloc": [ctypes.c_size_t, P, P],
        "bw_ipc_free": [P],
        "bw_ipc_open": [P, P],
        "bw_ipc_close": [P],
    }
    for name, args in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = I
    L.bw_last_error_string.argtypes = []
    L.bw_last_error_string.restype = ctypes.c_char_p
    L.bw_sf_bytes.argtypes = [I, I]
    L.bw_sf_bytes.restype = ctypes.c_size_t
    L.bw_sf_offset.argtypes = [I, I, I]
    L.bw_sf_offset.restype = ctypes.c_size_t
    _lib = L
    return L


def _check(rc: int) -> None:
    if rc != BW_OK:
        raise BwError(rc, lib().bw_last_error_string().decode(errors="replace"))


def _ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def _stream(stream) -> int | None:
    import torch

    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


# ------------------------------------------------------------------ runtime
def init(device: int = 0) -> None:
    _check(lib().bw_init(device))


def device_status(stream=None) -> int:
    out = ctypes.c_int(0)
    rc = lib().bw_device_status(_stream(stream), ctypes.byref(out))
    if rc not in (BW_OK, BW_ERR_TIMEOUT):
        _check(rc)
    return out.value


def set_wait_budget_ns(ns: int) -> None:
    _check(lib().bw_set_wait_budget_ns(int(ns)))


def set_trace_buffer(buf=None) -> None:
    """Arm the per-CTA wait-time trace with a torch int64 CUDA tensor of shape (ctas, 8)."""
    if buf is None:
        _check(lib().bw_set_trace_buffer(None, 0))
    else:
        _check(lib().bw_set_trace_buffer(buf.data_ptr(), buf.shape[0]))


def sf_bytes(outer: int, K: int) -> int:
    return int(lib().bw_sf_bytes(outer, K))


# ------------------------------------------------------------------ GEMMs
def gemm_f16(A, B, C=None, stream=None, b_transposed: bool = False):
    """C (fp32) = A (fp16 MxK) x B (fp16 KxN, or NxK when b_transposed)."""
    import torch

    M, K = A.shape
    N = B.shape[0] if b_transposed else B.shape[1]
    if C is None:
        C = torch.empty((M, N), dtype=torch.float32, device=A.device)
    fn = lib().bw_gemm_f16_bt if b_transposed else lib().bw_gemm_f16
    _check(fn(_ptr(A), _ptr(B), _ptr(C), M, N, K, _stream(stream)))
    return C


def gemm_fp8(A, Bt, scale_a=None, scale_b=None, C=None, out_dtype=OUT_BF16, stream=None):
    """C = (A (e4m3 MxK) x Bt^T (e4m3 NxK)) * scale_a * scale_b."""
    import torch

    M, K = A.shape
    N = Bt.shape[0]
    if C is None:
        C = torch.empty((M, N), dtype=torch.bfloat16 if out_dtype == OUT_BF16 else torch.float32, device=A.device)
    _check(lib().bw_gemm_fp8(_ptr(A), _ptr(Bt), _ptr(scale_a), _ptr(scale_b), _ptr(C), out_dtype, M, N, K,
                             _stream(stream)))
    return C


def gemm_mxfp4(A, Bt, sfa, sfb, K: int, scale_a=None, scale_b=None, C=None, out_dtype=OUT_BF16, stream=None):
    import torch

    M, N = A.shape[0], Bt.shape[0]
    if C is None:
        C = torch.empty((M, N), dtype=torch.bfloat16 if out_dtype == OUT_BF16 else torch.float32, device=A.device)
    _check(lib().bw_gemm_mxfp4(_ptr(A), _ptr(Bt), _ptr(sfa), _ptr(sfb), _ptr(scale_a), _ptr(scale_b), _ptr(C),
                               out_dtype, M, N, K, _stream(stream)))
    return C


def gemm_fp4(A, Bt, K: int, scale_a=None, scale_b=None, C=None, out_dtype=OUT_BF16, stream=None):
    import torch

    M, N = A.shape[0], Bt.shape[0]
    if C is None:
        C = torch.empty((M, N), dtype=torch.bfloat16 if out_dtype == OUT_BF16 else torch.float32, device=A.device)
    _check(lib().bw_gemm_fp4(_ptr(A), _ptr(Bt), _ptr(scale_a), _ptr(scale_b), _ptr(C), out_dtype, M, N, K,
                             _stream(stream)))
    return C


# ------------------------------------------------------------------ quantisers
def quantize_f16(src, dst=None, stream=None):
    import torch

    if dst is None:
        dst = torch.empty(src.shape, dtype=torch.float16, device=src.device)
    _check(lib().bw_quantize_f16(_ptr(src), _ptr(dst), src.numel(), _stream(stream)))
    return dst


def quantize_fp8(src, transpose=False, scale_mode=SCALE_AMAX, dst=None, scale_out=None, stream=None):
    import torch

    rows, cols = src.shape
    if dst is None:
        dst = torch.empty((cols, rows) if transpose else (rows, cols), dtype=torch.uint8, device=src.device)
    if scale_out is None:
        scale_out = torch.empty(1, dtype=torch.float32, device=src.device)
    _check(lib().bw_quantize_fp8(_ptr(src), _ptr(dst), _ptr(scale_out), rows, cols, int(transpose), scale_mode,
                                 _stream(stream)))
    return dst, scale_out


def quantize_fp8_noalloc(src, transpose=False, scale_mode=SCALE_AMAX, dst=None, scale_out=None, stream=None):
    """bw_quantize_fp8 through the entry point that allocates nothing (fixed library scratch).
    `dst` and `scale_out` must be supplied by callers that cannot allocate; the defaults here
    allocate them with torch for convenience."""
    import torch

    rows, cols = src.shape
    if dst is None:
        dst = torch.empty((cols, rows) if transpose else (rows, cols), dtype=torch.uint8, device=src.device)
    if scale_out is None:
        scale_out = torch.empty(1, dtype=torch.float32, device=src.device)
    _check(lib().bw_quantize_fp8_noalloc(_ptr(src), _ptr(dst), _ptr(scale_out), rows, cols, int(transpose),
                                         scale_mode, _stream(stream)))
    return dst, scale_out


def quantize_fp4(src, transpose=False, scale_mode=SCALE_AMAX, container=FP4_PACKED, dst=None, scale_out=None,
                 stream=None):
    import torch

    rows, cols = src.shape
    orows, ocols = (cols, rows) if transpose else (rows, cols)
    if dst is None:
        dst = torch.empty((orows, ocols if container == FP4_BYTE_SHL2 else ocols // 2), dtype=torch.uint8,
                          device=src.device)
    if scale_out is None:
        scale_out = torch.empty(1, dtype=torch.float32, device=src.device)
    _check(lib().bw_quantize_fp4(_ptr(src), _ptr(dst), _ptr(scale_out), rows, cols, int(transpose), scale_mode,
                                 container, _stream(stream)))
    return dst, scale_out


def quantize_mxfp4(src, transpose=False, mode=MX_BLOCK32, dst=None, sf=None, stream=None):
    import torch

    rows, cols = src.shape
    K, outer = (rows, cols) if transpose else (cols, rows)
    if dst is None:
        dst = torch.empty((outer, K // 2), dtype=torch.uint8, device=src.device)
    if sf is None:
        sf = torch.empty(sf_bytes(outer, K), dtype=torch.uint8, device=src.device)
    _check(lib().bw_quantize_mxfp4(_ptr(src), _ptr(dst), _ptr(sf), rows, cols, int(transpose), mode,
                                   _stream(stream)))
    return dst, sf


def unshard_columns(C_shardmajor, M: int, N: int, world: int, out=None, stream=None):
    """[world][M][N/world] -> row-major M x N on the device; FP32 or BF16 elements."""
    import torch

    if C_shardmajor.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"unshard_columns takes float32 or bfloat16, not {C_shardmajor.dtype}")
    if C_shardmajor.numel() != M * N:
        raise ValueError(f"shard-major buffer holds {C_shardmajor.numel()} elements, expected {M} x {N}")
    if out is None:
        out = torch.empty((M, N), dtype=C_shardmajor.dtype, device=C_shardmajor.device)
    if out.dtype != C_shardmajor.dtype or out.numel() != M * N:
        raise ValueError("out must match the input's dtype and hold M x N elements")
    fn = lib().bw_unshard_columns if C_shardmajor.dtype == torch.float32 else lib().bw_unshard_columns_bf16
    _check(fn(_ptr(C_shardmajor), _ptr(out), M, N, world, _stream(stream)))
    return out


def gemm_sharded(dtype: int, parts: list[dict], M: int, N: int, K: int, out_dtype: int = OUT_F32,
                 gather: bool = False) -> None:
    """One process, len(parts) GPUs: parts[r] = {"A", "B", "C", optional "sfA", "sfB", "scale_a",
    "scale_b", "C_gathered", "stream"} with torch tensors on the shard's device (B is the shard
    of columns r*N/g .. (r+1)*N/g in the layout of the dtype's single-GPU call). Enqueues the
    shards' GEMMs and, with gather, the NCCL all-gather + unshard into every C_gathered."""
    import torch

    arr = (Shard * max(1, len(parts)))()
    for r, part in enumerate(parts):
        dev = part["C"].device.index if part.get("C") is not None else 0
        st = part.get("stream")
        if st is None:
            st = torch.cuda.current_stream(dev)
        arr[r] = Shard(dev, _ptr(part.get("A")), _ptr(part.get("B")), _ptr(part.get("sfA")), _ptr(part.get("sfB")),
                       _ptr(part.get("scale_a")), _ptr(part.get("scale_b")), _ptr(part.get("C")),
                       _ptr(part.get("C_gathered")), _stream(st))
    _check(lib().bw_gemm_sharded(dtype, out_dtype, ctypes.cast(arr, ctypes.c_void_p) if parts else None,
                                 len(parts), M, N, K, int(gather)))


# ------------------------------------------------------------------ fused all-gather (IPC)
IPC_HANDLE_BYTES = 64


class IpcBuffer:
    """A device buffer other processes can map (CUDA IPC). `tensor` views it as a torch tensor
    (through __cuda_array_interface__, no copy); `handle` is the 64-byte IPC handle."""

    def __init__(self, shape, dtype, device):
        import math

        import torch

        self.shape, self.dtype = tuple(shape), dtype
        nbytes = math.prod(self.shape) * torch.empty((), dtype=dtype).element_size()
        ptr = ctypes.c_void_p()
        h = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        with torch.cuda.device(device):
            _check(lib().bw_ipc_malloc(nbytes, ctypes.byref(ptr), h))
        self.ptr, self.handle, self.device = ptr.value, h.raw, torch.device(device)
        typestr = {torch.float32: "<f4", torch.bfloat16: "<i2", torch.float16: "<f2"}[dtype]
        self.__cuda_array_interface__ = {"shape": self.shape, "typestr": typestr, "data": (self.ptr, False),
                                         "version": 3, "strides": None}
        t = torch.as_tensor(self, device=self.device)
        self.tensor = t.view(dtype) if dtype == torch.bfloat16 else t

    def close(self):
        if self.ptr:
            _check(lib().bw_ipc_free(self.ptr))
            self.ptr = None


def ipc_open(handle: bytes, device) -> int:
    import torch

    ptr = ctypes.c_void_p()
    with torch.cuda.device(device):
        _check(lib().bw_ipc_open(ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES), ctypes.byref(ptr)))
    return ptr.value


def ipc_close(ptr: int) -> None:
    _check(lib().bw_ipc_close(ptr))


def _peer_array(peers):
    return (ctypes.c_void_p * len(peers))(*[p or 0 for p in peers])


def gemm_f16_allgather(A, B_shard, C_full, peers, rank: int, stream=None):
    """This rank's columns of C_full = A x B_shard, stored locally and into every peer's C_full
    (peers[q] = rank q's buffer mapped here; entry [rank] ignored)."""
    M, K = A.shape
    world = len(peers)
    _check(lib().bw_gemm_f16_allgather(_ptr(A), _ptr(B_shard), _ptr(C_full), _peer_array(peers), world, rank, M,
                                       C_full.shape[1], K, _stream(stream)))


def gemm_fp8_allgather(A, Bt_shard, scale_a, scale_b, C_full, peers, rank: int, out_dtype=OUT_BF16, stream=None):
    M, K = A.shape
    world = len(peers)
    _check(lib().bw_gemm_fp8_allgather(_ptr(A), _ptr(Bt_shard), _ptr(scale_a), _ptr(scale_b), _ptr(C_full),
                                       out_dtype, _peer_array(peers), world, rank, M, C_full.shape[1], K,
                                       _stream(stream)))


def gemm_f16_allgather_multicast(A, B_shard, mc_ptr: int, world: int, rank: int, N_total: int, stream=None):
    """This rank's columns of the M x N_total product, written once through the multicast
    address `mc_ptr` (every rank's buffer bound to one NVLink multicast object) and so into
    every rank's C."""
    M, K = A.shape
    _check(lib().bw_gemm_f16_allgather_multicast(_ptr(A), _ptr(B_shard), mc_ptr, world, rank, M, N_total, K,
                                                 _stream(stream)))


def gemm_fp8_allgather_multicast(A, Bt_shard, scale_a, scale_b, mc_ptr: int, world: int, rank: int, N_total: int,
                                 out_dtype=OUT_BF16, stream=None):
    M, K = A.shape
    _check(lib().bw_gemm_fp8_allgather_multicast(_ptr(A), _ptr(Bt_shard), _ptr(scale_a), _ptr(scale_b), mc_ptr,
                                                 out_dtype, world, rank, M, N_total, K, _stream(stream)))
