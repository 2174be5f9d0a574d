"""Python binding of libbsp.so (the C ABI in include/bsp.h), via ctypes.

Device memory comes from torch tensors (torch is plumbing here: allocation,
streams, NCCL); every multiply runs in libbsp's sm_100a kernels.  There is no
CPU or torch fallback: if libbsp.so is missing or the call fails, this raises.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libbsp.so")

BSP_OK, BSP_ERR_INVALID_ARG, BSP_ERR_UNSUPPORTED, BSP_ERR_CUDA, BSP_ERR_TIMEOUT = 0, 1, 2, 3, 4
NAIVE, SNF, DDA = 0, 1, 2
BF16, F32 = 0, 1
STRATEGIES = {"naive": NAIVE, "snf": SNF, "dda": DDA}

# Every symbol the header declares (checked by the CPU test suite).
EXPORTS = [
    "bsp_device_open", "bsp_device_close", "bsp_device_synchronize", "bsp_device_get_error",
    "bsp_device_sm_count", "bsp_last_error_string", "bsp_status_string",
    "bsp_spmm_plan_create", "bsp_spmm_execute", "bsp_spmm_plan_destroy", "bsp_spmm_plan_info",
    "bsp_spmm", "bsp_spmm_host",
    "bsp_sddmm_plan_create", "bsp_sddmm_execute", "bsp_sddmm_plan_destroy",
    "bsp_sddmm_plan_info", "bsp_sddmm", "bsp_sddmm_host",
    "bsp_partition_rows", "bsp_serpentine_assign", "bsp_spmm_host_profile",
    "bsp_sddmm_host_profile", "bsp_spmm_plan_inspect", "bsp_sddmm_plan_inspect",
    "bsp_spmm_noalloc", "bsp_spmm_execute_replicated", "bsp_ipc_export", "bsp_ipc_import",
    "bsp_ipc_close", "bsp_spgemm_plan_create", "bsp_spgemm_pattern", "bsp_spgemm_execute",
    "bsp_spgemm_plan_destroy", "bsp_spgemm_plan_info", "bsp_spgemm_host", "bsp_spgemm_plan_inspect",
    "bsp_attn_plan_create", "bsp_attn_execute", "bsp_attn_plan_destroy", "bsp_attn_plan_info",
    "bsp_attn_host", "bsp_attn_plan_inspect", "bsp_spmm_plan_traffic", "bsp_spmm_plan_entry_rows",
]
IPC_HANDLE_BYTES = 64


class BspError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"bsp error {status}: {msg}")
        self.status = status


class BsrDesc(ctypes.Structure):
    _fields_ = [
        ("rows", ctypes.c_int64), ("cols", ctypes.c_int64),
        ("R", ctypes.c_int32), ("C", ctypes.c_int32),
        ("nnzb", ctypes.c_int64),
        ("row_ptr", ctypes.c_void_p), ("col_idx", ctypes.c_void_p), ("values", ctypes.c_void_p),
    ]


class SpmmHostJob(ctypes.Structure):
    """bsp_spmm_host_job: one product of bsp_spmm_host_batch (host arrays)."""
    _fields_ = [
        ("M", ctypes.c_int64), ("K", ctypes.c_int64), ("R", ctypes.c_int32), ("C", ctypes.c_int32),
        ("nnzb", ctypes.c_int64), ("row_ptr", ctypes.c_void_p), ("col_idx", ctypes.c_void_p),
        ("values", ctypes.c_void_p), ("B", ctypes.c_void_p), ("N", ctypes.c_int64), ("C_out", ctypes.c_void_p),
    ]


class Opts(ctypes.Structure):
    _fields_ = [
        ("no_load_balance", ctypes.c_int32), ("group_rows", ctypes.c_int32),
        ("n_tiles", ctypes.c_int32), ("max_ctas", ctypes.c_int32),
        ("timeout_ms", ctypes.c_int32), ("group_mma", ctypes.c_int32),
        ("producers", ctypes.c_int32), ("steps_per_stage", ctypes.c_int32),
    ]


_lib = None


def lib():
    """Load libbsp.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"libbsp.so not built at {LIB_PATH}; run __graft_entry__.build()")
    L = ctypes.CDLL(LIB_PATH)
    P, I64, I32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
    S = ctypes.c_int
    sig = {
        "bsp_device_open": (S, [ctypes.c_int, ctypes.POINTER(P)]),
        "bsp_device_close": (S, [P]),
        "bsp_device_synchronize": (S, [P]),
        "bsp_device_get_error": (S, [P, ctypes.POINTER(ctypes.c_uint32)]),
        "bsp_device_sm_count": (ctypes.c_int, [P]),
        "bsp_last_error_string": (ctypes.c_char_p, []),
        "bsp_status_string": (ctypes.c_char_p, [S]),
        "bsp_spmm_plan_create": (S, [P, ctypes.POINTER(BsrDesc), P, P, I64, S, S,
                                     ctypes.POINTER(Opts), ctypes.POINTER(P)]),
        "bsp_spmm_execute": (S, [P, ctypes.POINTER(BsrDesc), P, I64, P, I64, P]),
        "bsp_spmm_plan_destroy": (S, [P]),
        "bsp_spmm_plan_info": (S, [P, ctypes.POINTER(I64)]),
        "bsp_spmm": (S, [P, ctypes.POINTER(BsrDesc), P, I64, P, I64, S, I64, S,
                         ctypes.POINTER(Opts), P]),
        "bsp_spmm_host": (S, [P, I64, I64, I32, I32, I64, P, P, P, P, I64, P, S,
                              ctypes.POINTER(Opts)]),
        "bsp_sddmm_plan_create": (S, [P, ctypes.POINTER(BsrDesc), P, P, I64, S,
                                      ctypes.POINTER(Opts), ctypes.POINTER(P)]),
        "bsp_sddmm_execute": (S, [P, ctypes.POINTER(BsrDesc), P, I64, P, I64, P, P]),
        "bsp_sddmm_plan_destroy": (S, [P]),
        "bsp_sddmm_plan_info": (S, [P, ctypes.POINTER(I64)]),
        "bsp_sddmm": (S, [P, ctypes.POINTER(BsrDesc), P, I64, P, I64, I64, P, S,
                          ctypes.POINTER(Opts), P]),
        "bsp_sddmm_host": (S, [P, I64, I64, I32, I32, I64, P, P, P, P, P, I64, P, S,
                               ctypes.POINTER(Opts)]),
        "bsp_partition_rows": (S, [P, I64, I32, P]),
        "bsp_serpentine_assign": (S, [I64, I32, P, P]),
        "bsp_spmm_host_profile": (S, [P, I64, I64, I32, I32, I64, P, P, P, P, I64, P, S,
                                      ctypes.POINTER(Opts), I32, ctypes.POINTER(ctypes.c_double)]),
        "bsp_sddmm_host_profile": (S, [P, I64, I64, I32, I32, I64, P, P, P, P, P, I64, P, S,
                                       ctypes.POINTER(Opts), I32, ctypes.POINTER(ctypes.c_double)]),
        "bsp_spmm_plan_inspect": (S, [I64, I64, I32, I32, I64, P, P, I64, S, S, ctypes.POINTER(Opts),
                                      I32, I32, P, P, P, P, P, P]),
        "bsp_spmm_noalloc": (S, [ctypes.POINTER(BsrDesc), P, P, P, I64, P, I64, I64, S, S, P]),
        "bsp_spmm_execute_replicated": (S, [P, ctypes.POINTER(BsrDesc), P, I64, P, I64,
                                            ctypes.POINTER(ctypes.c_void_p), I32, P]),
        "bsp_ipc_export": (S, [P, P, P, ctypes.POINTER(ctypes.c_int64)]),
        "bsp_ipc_import": (S, [P, P, ctypes.POINTER(ctypes.c_void_p)]),
        "bsp_ipc_close": (S, [P, P]),
        "bsp_sddmm_plan_inspect": (S, [I64, I64, I32, I32, I64, P, P, I64, S, ctypes.POINTER(Opts),
                                       I32, I32, P, P, P]),
        "bsp_spgemm_plan_create": (S, [P, ctypes.POINTER(BsrDesc), P, P, ctypes.POINTER(BsrDesc),
                                       P, P, ctypes.POINTER(Opts), ctypes.POINTER(P)]),
        "bsp_spgemm_pattern": (S, [P, ctypes.POINTER(I64), P, P]),
        "bsp_spgemm_execute": (S, [P, ctypes.POINTER(BsrDesc), ctypes.POINTER(BsrDesc), P, P]),
        "bsp_spgemm_plan_destroy": (S, [P]),
        "bsp_spgemm_plan_info": (S, [P, ctypes.POINTER(I64)]),
        "bsp_spgemm_host": (S, [P, I64, I64, I64, I32, I32, I32, I64, P, P, P, I64, P, P, P, I64,
                                ctypes.POINTER(I64), P, P, P, ctypes.POINTER(Opts), I32,
                                ctypes.POINTER(ctypes.c_double)]),
        "bsp_spgemm_plan_inspect": (S, [I64, I64, I64, I32, I32, I32, I64, P, P, I64, P, P,
                                        ctypes.POINTER(Opts), I32, I32, P, P, P, P, P, P]),
        "bsp_attn_plan_create": (S, [P, ctypes.POINTER(BsrDesc), P, P, I64, ctypes.POINTER(Opts),
                                     ctypes.POINTER(P)]),
        "bsp_attn_execute": (S, [P, P, I64, P, I64, P, I64, ctypes.c_float, P, I64, P]),
        "bsp_attn_plan_destroy": (S, [P]),
        "bsp_attn_plan_info": (S, [P, ctypes.POINTER(I64)]),
        "bsp_attn_host": (S, [P, I64, I64, I64, P, P, P, P, P, ctypes.c_float, P, ctypes.POINTER(Opts)]),
        "bsp_attn_plan_inspect": (S, [I64, I64, I64, P, P, ctypes.POINTER(Opts), I32, I32, P, P, P, P]),
        "bsp_spmm_plan_traffic": (S, [I64, I64, I32, I32, I64, P, P, I64, S, ctypes.POINTER(Opts), I32, I32,
                                      P, P]),
        "bsp_spmm_plan_entry_rows": (S, [I64, I64, I32, I32, I64, P, P, I64, S, ctypes.POINTER(Opts), I32, I32,
                                         P, ctypes.POINTER(I64)]),
        "bsp_testing_spmm_counters": (S, [P, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(I64),
                                          ctypes.POINTER(I32)]),
        "bsp_testing_spmm_drop_stage": (S, [P, I32]),
        "bsp_spmm_host_batch": (S, [P, I32, ctypes.POINTER(SpmmHostJob), S, ctypes.POINTER(Opts)]),
        "bsp_bsr_upload": (S, [P, I64, I64, I32, I32, I64, P, P, P, ctypes.POINTER(BsrDesc)]),
        "bsp_bsr_free": (S, [P, ctypes.POINTER(BsrDesc)]),
        "bsp_buffer_alloc": (S, [P, I64, ctypes.POINTER(ctypes.c_void_p)]),
        "bsp_buffer_free": (S, [P, P]),
        "bsp_buffer_write": (S, [P, P, P, I64]),
        "bsp_buffer_read": (S, [P, P, P, I64]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _check(status: int):
    if status != BSP_OK:
        raise BspError(status, lib().bsp_last_error_string().decode())


def make_opts(**kw) -> Opts:
    o = Opts()
    for k, v in kw.items():
        if v is not None:
            setattr(o, k, int(v))
    return o


def _ptr(a) -> Optional[int]:
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


# ------------------------------------------------------------------ device --
class Device:
    """A B200 (sm_100a) opened through the library (reference: IDevice*)."""

    def __init__(self, ordinal: int = 0):
        h = ctypes.c_void_p()
        _check(lib().bsp_device_open(ordinal, ctypes.byref(h)))
        self.handle = h
        self.ordinal = ordinal

    @property
    def sm_count(self) -> int:
        return lib().bsp_device_sm_count(self.handle)

    def synchronize(self):
        _check(lib().bsp_device_synchronize(self.handle))

    def status_bits(self) -> int:
        v = ctypes.c_uint32()
        _check(lib().bsp_device_get_error(self.handle, ctypes.byref(v)))
        return v.value

    def close(self):
        if self.handle:
            lib().bsp_device_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_default = {}


def device(ordinal: int = 0) -> Device:
    if ordinal not in _default:
        _default[ordinal] = Device(ordinal)
    return _default[ordinal]


# ---------------------------------------------------------------- BSR data --
@dataclass
class DeviceBSR:
    """A BSR matrix resident on the GPU (torch tensors) plus its host pattern."""

    rows: int
    cols: int
    R: int
    C: int
    row_ptr: "object"   # torch int32 cuda
    col_idx: "object"   # torch int32 cuda
    values: "object"    # torch bf16 cuda, [nnzb*R*C] (or None for a pattern-only mask)
    h_row_ptr: np.ndarray
    h_col_idx: np.ndarray

    @property
    def nnzb(self) -> int:
        return int(self.h_row_ptr[-1])

    def desc(self) -> BsrDesc:
        return BsrDesc(self.rows, self.cols, self.R, self.C, self.nnzb,
                       _ptr(self.row_ptr), _ptr(self.col_idx), _ptr(self.values))

    @staticmethod
    def from_host(rows, cols, R, C, row_ptr, col_idx, values_bf16_bits=None, device_index=0):
        import torch
        dev = torch.device("cuda", device_index)
        rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
        ci = np.ascontiguousarray(col_idx, dtype=np.int32)
        t_rp = torch.from_numpy(rp).to(dev)
        t_ci = torch.from_numpy(ci if ci.size else np.zeros(1, np.int32)).to(dev)
        t_v = None
        if values_bf16_bits is not None:
            v = np.ascontiguousarray(values_bf16_bits, dtype=np.uint16).ravel()
            if v.size == 0:
                v = np.zeros(8, np.uint16)
            t_v = torch.from_numpy(v.view(np.int16)).to(dev).view(torch.bfloat16)
        return DeviceBSR(rows, cols, R, C, t_rp, t_ci, t_v, rp, ci)


def to_device_bf16(bits: np.ndarray, device_index=0):
    import torch
    a = np.ascontiguousarray(bits, dtype=np.uint16)
    return torch.from_numpy(a.view(np.int16)).to(torch.device("cuda", device_index)).view(torch.bfloat16)


def to_host_bits(t) -> np.ndarray:
    import torch
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _stream_ptr(stream) -> Optional[int]:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


# -------------------------------------------------------------------- SpMM --
class SpmmPlan:
    """Reusable SpMM plan for one pattern and one N (reference: the planner)."""

    def __init__(self, dev: Device, A: DeviceBSR, N: int, strategy=NAIVE, c_type=BF16, opts=None):
        self.dev, self.N, self.c_type = dev, N, c_type
        self._desc = A.desc()
        h = ctypes.c_void_p()
        o = opts if opts is not None else Opts()
        _check(lib().bsp_spmm_plan_create(dev.handle, ctypes.byref(self._desc),
                                          _ptr(A.h_row_ptr), _ptr(A.h_col_idx), N, c_type,
                                          strategy, ctypes.byref(o), ctypes.byref(h)))
        self.handle = h

    def info(self) -> dict:
        arr = (ctypes.c_int64 * 16)()
        _check(lib().bsp_spmm_plan_info(self.handle, arr))
        keys = ["units", "ctas", "group_rows", "n_tiles", "slab", "kc", "stages", "steps",
                "plan_bytes", "smem_bytes", "tmem_cols", "variant", "producers"]
        return {k: int(arr[i]) for i, k in enumerate(keys)}

    def execute(self, A: DeviceBSR, B, C, stream=None):
        d = A.desc()
        _check(lib().bsp_spmm_execute(self.handle, ctypes.byref(d), _ptr(B), B.stride(0), _ptr(C),
                                      C.stride(0), _stream_ptr(stream)))

    def execute_replicated(self, A: DeviceBSR, B, C, peer_ptrs, stream=None):
        """execute(), and every C store repeated into the peers' C buffers
        (device pointers of the element matching C[0][0] on each peer)."""
        d = A.desc()
        arr = (ctypes.c_void_p * max(len(peer_ptrs), 1))(*[int(x) for x in peer_ptrs])
        _check(lib().bsp_spmm_execute_replicated(self.handle, ctypes.byref(d), _ptr(B), B.stride(0),
                                                 _ptr(C), C.stride(0), arr, len(peer_ptrs),
                                                 _stream_ptr(stream)))

    def close(self):
        if self.handle:
            lib().bsp_spmm_plan_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def spmm(A: DeviceBSR, B, strategy=NAIVE, c_type=BF16, opts=None, dev: Device = None):
    """One-shot C = A @ B on the GPU (B: torch bf16 cuda [K, N]); returns C."""
    import torch
    dev = dev or device(B.device.index or 0)
    N = B.shape[1]
    C = torch.empty((A.rows, N), dtype=torch.float32 if c_type == F32 else torch.bfloat16,
                    device=B.device)
    plan = SpmmPlan(dev, A, N, strategy, c_type, opts)
    plan.execute(A, B, C)
    dev.synchronize()
    plan.close()
    return C


def spmm_host(M, K, R, C, row_ptr, col_idx, values, B, N, strategy=NAIVE, opts=None,
              dev: Device = None, out=None) -> np.ndarray:
    """Host buffers in, host C out (reference planner semantics)."""
    dev = dev or device(0)
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    ci = np.ascontiguousarray(col_idx, dtype=np.int32)
    v = np.ascontiguousarray(values, dtype=np.uint16)
    b = np.ascontiguousarray(B, dtype=np.uint16)
    o = out if out is not None else np.empty((M, N), dtype=np.uint16)
    opt = opts if opts is not None else Opts()
    _check(lib().bsp_spmm_host(dev.handle, M, K, R, C, int(rp[-1]), _ptr(rp), _ptr(ci), _ptr(v),
                               _ptr(b), N, _ptr(o), strategy, ctypes.byref(opt)))
    return o


def spmm_host_batch(jobs, strategy=NAIVE, opts=None, dev: Device = None):
    """Several host-buffer SpMMs in one pipelined call (bsp_spmm_host_batch).
    jobs: sequence of dicts with M, K, R, C, row_ptr, col_idx, values, B, N and
    optionally out (a uint16 M x N array to write); returns the outputs."""
    dev = dev or device(0)
    keep, arr = [], (SpmmHostJob * max(len(jobs), 1))()
    outs = []
    for k, j in enumerate(jobs):
        rp = np.ascontiguousarray(j["row_ptr"], dtype=np.int32)
        ci = np.ascontiguousarray(j["col_idx"], dtype=np.int32)
        v = np.ascontiguousarray(j["values"], dtype=np.uint16)
        b = np.ascontiguousarray(j["B"], dtype=np.uint16)
        o = j.get("out")
        if o is None:
            o = np.empty((j["M"], j["N"]), dtype=np.uint16)
        keep += [rp, ci, v, b, o]
        outs.append(o)
        arr[k] = SpmmHostJob(j["M"], j["K"], j["R"], j["C"], int(rp[-1]), _ptr(rp), _ptr(ci), _ptr(v), _ptr(b),
                             j["N"], _ptr(o))
    opt = opts if opts is not None else Opts()
    _check(lib().bsp_spmm_host_batch(dev.handle, len(jobs), arr, strategy, ctypes.byref(opt)))
    return outs


# ------------------------------------------------------------------- SDDMM --
class SddmmPlan:
    def __init__(self, dev: Device, mask: DeviceBSR, K: int, strategy=NAIVE, opts=None):
        self.dev, self.K = dev, K
        self._desc = mask.desc()
        h = ctypes.c_void_p()
        o = opts if opts is not None else Opts()
        _check(lib().bsp_sddmm_plan_create(dev.handle, ctypes.byref(self._desc),
                                           _ptr(mask.h_row_ptr), _ptr(mask.h_col_idx), K,
                                           strategy, ctypes.byref(o), ctypes.byref(h)))
        self.handle = h

    def info(self) -> dict:
        arr = (ctypes.c_int64 * 16)()
        _check(lib().bsp_sddmm_plan_info(self.handle, arr))
        keys = ["units", "ctas", "_2", "_3", "slab", "kc", "stages", "keep_a", "plan_bytes",
                "smem_bytes", "tmem_cols", "variant", "_12", "nseg_max", "producers"]
        return {k: int(arr[i]) for i, k in enumerate(keys) if not k.startswith("_")}

    def execute(self, mask: DeviceBSR, A, B, out, stream=None):
        d = mask.desc()
        _check(lib().bsp_sddmm_execute(self.handle, ctypes.byref(d), _ptr(A), A.stride(0), _ptr(B),
                                       B.stride(0), _ptr(out), _stream_ptr(stream)))

    def close(self):
        if self.handle:
            lib().bsp_sddmm_plan_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def sddmm(mask: DeviceBSR, A, B, strategy=NAIVE, opts=None, dev: Device = None):
    """One-shot out = mask (.) (A @ B) on the mask's pattern; returns bf16 block values."""
    import torch
    dev = dev or device(A.device.index or 0)
    out = torch.empty(max(mask.nnzb * mask.R * mask.C, 8), dtype=torch.bfloat16, device=A.device)
    plan = SddmmPlan(dev, mask, A.shape[1], strategy, opts)
    plan.execute(mask, A, B, out)
    dev.synchronize()
    plan.close()
    return out[: mask.nnzb * mask.R * mask.C]


def sddmm_host(M, N, R, C, row_ptr, col_idx, mask_values, A, B, K, strategy=NAIVE, opts=None,
               dev: Device = None, out=None) -> np.ndarray:
    dev = dev or device(0)
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    ci = np.ascontiguousarray(col_idx, dtype=np.int32)
    mv = None if mask_values is None else np.ascontiguousarray(mask_values, dtype=np.uint16)
    a = np.ascontiguousarray(A, dtype=np.uint16)
    b = np.ascontiguousarray(B, dtype=np.uint16)
    nnzb = int(rp[-1])
    o = out if out is not None else np.empty(nnzb * R * C, dtype=np.uint16)
    opt = opts if opts is not None else Opts()
    _check(lib().bsp_sddmm_host(dev.handle, M, N, R, C, nnzb, _ptr(rp), _ptr(ci), _ptr(mv),
                                _ptr(a), _ptr(b), K, _ptr(o), strategy, ctypes.byref(opt)))
    return o


# ------------------------------------------------------------------ SpGEMM --
SPGEMM_INFO_KEYS = ["units", "ctas", "steps", "pairs", "out_nnzb", "kc", "stages",
                    "steps_per_stage", "plan_bytes", "smem_bytes", "tmem_cols", "nseg_max",
                    "producers", "boxes"]


class SpgemmPlan:
    """C = A @ B for two BSR matrices (bsr_matrix<T>::spgemm,
    sparse_common/bsr_matrix.hpp:741-810); the plan holds C's pattern."""

    def __init__(self, dev: Device, A: DeviceBSR, B: DeviceBSR, opts=None):
        self.dev = dev
        self.M, self.N, self.Ra, self.Cb = A.rows, B.cols, A.R, B.C
        da, db = A.desc(), B.desc()
        h = ctypes.c_void_p()
        o = opts if opts is not None else Opts()
        _check(lib().bsp_spgemm_plan_create(dev.handle, ctypes.byref(da), _ptr(A.h_row_ptr),
                                            _ptr(A.h_col_idx), ctypes.byref(db), _ptr(B.h_row_ptr),
                                            _ptr(B.h_col_idx), ctypes.byref(o), ctypes.byref(h)))
        self.handle = h
        n = ctypes.c_int64()
        _check(lib().bsp_spgemm_pattern(h, ctypes.byref(n), None, None))
        self.nnzb = int(n.value)
        self.row_ptr = np.zeros(self.M // self.Ra + 1, np.int32)
        self.col_idx = np.zeros(max(self.nnzb, 1), np.int32)
        _check(lib().bsp_spgemm_pattern(h, ctypes.byref(n), _ptr(self.row_ptr), _ptr(self.col_idx)))
        self.col_idx = self.col_idx[: self.nnzb]

    def info(self) -> dict:
        arr = (ctypes.c_int64 * 16)()
        _check(lib().bsp_spgemm_plan_info(self.handle, arr))
        return {k: int(arr[i]) for i, k in enumerate(SPGEMM_INFO_KEYS)}

    def execute(self, A: DeviceBSR, B: DeviceBSR, out, stream=None):
        """out: device bf16, at least nnzb * Ra * Cb elements."""
        da, db = A.desc(), B.desc()
        _check(lib().bsp_spgemm_execute(self.handle, ctypes.byref(da), ctypes.byref(db), _ptr(out),
                                        _stream_ptr(stream)))

    def close(self):
        if self.handle:
            lib().bsp_spgemm_plan_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def spgemm(A: DeviceBSR, B: DeviceBSR, opts=None, dev: Device = None) -> DeviceBSR:
    """One-shot C = A @ B (both BSR on the GPU); returns C as a DeviceBSR."""
    import torch
    dev = dev or device(A.values.device.index or 0)
    plan = SpgemmPlan(dev, A, B, opts)
    out = torch.empty(max(plan.nnzb * A.R * B.C, 8), dtype=torch.bfloat16, device=A.values.device)
    plan.execute(A, B, out)
    dev.synchronize()
    C = DeviceBSR(A.rows, B.cols, A.R, B.C,
                  torch.from_numpy(plan.row_ptr.copy()).to(out.device),
                  torch.from_numpy(plan.col_idx.copy() if plan.nnzb else np.zeros(1, np.int32)).to(out.device),
                  out, plan.row_ptr.copy(), plan.col_idx.copy())
    plan.close()
    return C


def spgemm_host(M, K, N, Ra, Ca, Cb, a_row_ptr, a_col_idx, a_values, b_row_ptr, b_col_idx,
                b_values, opts=None, dev: Device = None, iters=0):
    """Host BSR in, host BSR out: (row_ptr, col_idx, values bf16 bits) of A @ B
    (bsr_matrix<T>::spgemm semantics), plus the mean launch time in ms when
    iters > 0.  Uploads, plans once (C's pattern on the host), runs, downloads."""
    import torch

    dev = dev or device(0)
    A = DeviceBSR.from_host(M, K, Ra, Ca, a_row_ptr, a_col_idx, a_values, dev.ordinal)
    B = DeviceBSR.from_host(K, N, Ca, Cb, b_row_ptr, b_col_idx, b_values, dev.ordinal)
    plan = SpgemmPlan(dev, A, B, opts)
    n = plan.nnzb * Ra * Cb
    out = torch.empty(max(n, 8), dtype=torch.bfloat16, device=A.row_ptr.device)
    plan.execute(A, B, out)
    ms = 0.0
    if iters > 0:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            plan.execute(A, B, out)
        e1.record()
        e1.synchronize()
        ms = e0.elapsed_time(e1) / iters
    dev.synchronize()
    res = (plan.row_ptr.copy(), plan.col_idx.copy(), to_host_bits(out)[:n])
    plan.close()
    return res + (ms,) if iters > 0 else res


def spgemm_host_c(M, K, N, Ra, Ca, Cb, a_row_ptr, a_col_idx, a_values, b_row_ptr, b_col_idx,
                  b_values, opts=None, dev: Device = None, iters=0):
    """The same through the C ABI's host-buffer entry point bsp_spgemm_host
    (a size query, then the product: C's pattern is planned twice)."""
    dev = dev or device(0)
    arp = np.ascontiguousarray(a_row_ptr, dtype=np.int32)
    aci = np.ascontiguousarray(a_col_idx, dtype=np.int32)
    av = np.ascontiguousarray(a_values, dtype=np.uint16)
    brp = np.ascontiguousarray(b_row_ptr, dtype=np.int32)
    bci = np.ascontiguousarray(b_col_idx, dtype=np.int32)
    bv = np.ascontiguousarray(b_values, dtype=np.uint16)
    opt = opts if opts is not None else Opts()
    n = ctypes.c_int64()
    ms = ctypes.c_double(0.0)
    common = (dev.handle, M, K, N, Ra, Ca, Cb, int(arp[-1]), _ptr(arp), _ptr(aci), _ptr(av),
              int(brp[-1]), _ptr(brp), _ptr(bci), _ptr(bv))
    _check(lib().bsp_spgemm_host(*common, 0, ctypes.byref(n), None, None, None, ctypes.byref(opt),
                                 0, None))
    cap = int(n.value)
    orp = np.zeros(M // Ra + 1, np.int32)
    oci = np.zeros(max(cap, 1), np.int32)
    ov = np.zeros(max(cap * Ra * Cb, 8), np.uint16)
    _check(lib().bsp_spgemm_host(*common, cap, ctypes.byref(n), _ptr(orp), _ptr(oci), _ptr(ov),
                                 ctypes.byref(opt), iters, ctypes.byref(ms)))
    res = (orp, oci[:cap], ov[: cap * Ra * Cb])
    return res + (ms.value,) if iters > 0 else res


def inspect_spgemm_plan(M, K, N, Ra, Ca, Cb, a_row_ptr, a_col_idx, b_row_ptr, b_col_idx, opts=None,
                        sm_count=148, max_smem=232448):
    """Run the SpGEMM planner on the host only (no GPU) and return its schedule."""
    arp = np.ascontiguousarray(a_row_ptr, dtype=np.int32)
    aci = np.ascontiguousarray(a_col_idx, dtype=np.int32)
    brp = np.ascontiguousarray(b_row_ptr, dtype=np.int32)
    bci = np.ascontiguousarray(b_col_idx, dtype=np.int32)
    aci = aci if aci.size else np.zeros(1, np.int32)
    bci = bci if bci.size else np.zeros(1, np.int32)
    info = np.zeros(16, np.int64)
    o = opts if opts is not None else Opts()
    args = (M, K, N, Ra, Ca, Cb, int(arp[-1]), _ptr(arp), _ptr(aci), int(brp[-1]), _ptr(brp),
            _ptr(bci), ctypes.byref(o), sm_count, max_smem, _ptr(info))
    _check(lib().bsp_spgemm_plan_inspect(*args, None, None, None, None, None))
    nu, ns, nb, nc = int(info[0]), int(info[2]), int(info[4]), int(info[1])
    orp = np.zeros(M // Ra + 1, np.int32)
    oci = np.zeros(max(nb, 1), np.int32)
    units = np.zeros((max(nu, 1), 48), np.int32)
    steps = np.zeros((max(ns, 1), 16), np.int32)
    cta = np.zeros(nc + 1, np.int32)
    _check(lib().bsp_spgemm_plan_inspect(*args, _ptr(orp), _ptr(oci), _ptr(units), _ptr(steps),
                                         _ptr(cta)))
    d = {k: int(info[i]) for i, k in enumerate(SPGEMM_INFO_KEYS)}
    d.update(out_row_ptr=orp, out_col_idx=oci[:nb], unit_table=units[:nu], step_table=steps[:ns],
             cta_begin=cta)
    return d


# --------------------------------------------------------------- attention --
ATTN_INFO_KEYS = ["units", "ctas", "chunks", "mask_blocks", "S", "d", "parts", "split_units",
                  "plan_bytes", "smem_bytes", "tmem_cols"]


class AttnPlan:
    """Fused block-sparse attention step for one mask pattern and head size:
    O = softmax_rows(scale * Q K^T on the mask's blocks) V (the reference's
    SDDMM -> softmax -> SpMM chain in one kernel)."""

    def __init__(self, dev: Device, mask: DeviceBSR, d: int, opts=None):
        self.dev, self.d, self.S = dev, d, mask.rows
        self._desc = mask.desc()
        h = ctypes.c_void_p()
        o = opts if opts is not None else Opts()
        _check(lib().bsp_attn_plan_create(dev.handle, ctypes.byref(self._desc), _ptr(mask.h_row_ptr),
                                          _ptr(mask.h_col_idx), d, ctypes.byref(o), ctypes.byref(h)))
        self.handle = h

    def info(self) -> dict:
        arr = (ctypes.c_int64 * 16)()
        _check(lib().bsp_attn_plan_info(self.handle, arr))
        return {k: int(arr[i]) for i, k in enumerate(ATTN_INFO_KEYS) if not k.startswith("_")}

    def execute(self, Q, K, V, O, scale=None, stream=None):
        """Q, K, V, O: torch bf16 cuda [S, d] (row strides may exceed d)."""
        sc = float(scale) if scale is not None else 1.0 / float(np.sqrt(self.d))
        _check(lib().bsp_attn_execute(self.handle, _ptr(Q), Q.stride(0), _ptr(K), K.stride(0), _ptr(V),
                                      V.stride(0), sc, _ptr(O), O.stride(0), _stream_ptr(stream)))

    def close(self):
        if self.handle:
            lib().bsp_attn_plan_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def attention(mask: DeviceBSR, Q, K, V, scale=None, opts=None, dev: Device = None):
    """One-shot fused attention step on device tensors; returns O."""
    import torch

    dev = dev or device(Q.device.index or 0)
    O = torch.empty_like(Q)
    plan = AttnPlan(dev, mask, Q.shape[1], opts)
    plan.execute(Q, K, V, O, scale)
    dev.synchronize()
    plan.close()
    return O


def attn_host(S, d, row_ptr, col_idx, Q, K, V, scale=None, opts=None, dev: Device = None):
    """Host arrays in (pattern, Q, K, V bf16 bits), host O out (bsp_attn_host)."""
    dev = dev or device(0)
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    ci = np.ascontiguousarray(col_idx, dtype=np.int32)
    q = np.ascontiguousarray(Q, dtype=np.uint16)
    k = np.ascontiguousarray(K, dtype=np.uint16)
    v = np.ascontiguousarray(V, dtype=np.uint16)
    o = np.empty((S, d), dtype=np.uint16)
    sc = float(scale) if scale is not None else 1.0 / float(np.sqrt(d))
    opt = opts if opts is not None else Opts()
    _check(lib().bsp_attn_host(dev.handle, S, d, int(rp[-1]), _ptr(rp), _ptr(ci), _ptr(q), _ptr(k), _ptr(v),
                               sc, _ptr(o), ctypes.byref(opt)))
    return o


def inspect_attn_plan(S, d, row_ptr, col_idx, opts=None, sm_count=148, max_smem=232448):
    """Run the attention planner on the host only (no GPU)."""
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    ci = np.ascontiguousarray(col_idx, dtype=np.int32)
    ci = ci if ci.size else np.zeros(1, np.int32)
    info = np.zeros(16, np.int64)
    o = opts if opts is not None else Opts()
    args = (S, d, int(rp[-1]), _ptr(rp), _ptr(ci), ctypes.byref(o), sm_count, max_smem, _ptr(info))
    _check(lib().bsp_attn_plan_inspect(*args, None, None, None))
    units = np.zeros((max(int(info[0]), 1), 8), np.int32)
    chunks = np.zeros((max(int(info[2]), 1), 8), np.int32)
    cta = np.zeros(int(info[1]) + 1, np.int32)
    _check(lib().bsp_attn_plan_inspect(*args, _ptr(units), _ptr(chunks), _ptr(cta)))
    dd = {k: int(info[i]) for i, k in enumerate(ATTN_INFO_KEYS) if not k.startswith("_")}
    dd.update(unit_table=units[: int(info[0])], chunk_table=chunks[: int(info[2])], cta_begin=cta)
    return dd


# ----------------------------------------------------------------- helpers --
def inspect_spmm_plan(M, K, R, C, row_ptr, col_idx, N, strategy=NAIVE, c_type=BF16, opts=None,
                      sm_count=148, max_smem=232448):
    """Run the SpMM planner on the host only (no GPU) and return its schedule."""
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    ci = np.ascontiguousarray(col_idx, dtype=np.int32)
    if ci.size == 0:
        ci = np.zeros(1, np.int32)
    info = np.zeros(16, np.int64)
    o = opts if opts is not None else Opts()
    args = (M, K, R, C, int(rp[-1]), _ptr(rp), _ptr(ci), N, c_type, strategy, ctypes.byref(o),
            sm_count, max_smem, _ptr(info))
    _check(lib().bsp_spmm_plan_inspect(*args, None, None, None, None, None))
    units = np.zeros((int(info[0]), 8), np.int32)
    cta = np.zeros(int(info[1]) + 1, np.int32)
    steps = np.zeros((max(int(info[7]), 1), int(info[15])), np.int32)
    stages = np.zeros((max(int(info[13]), 1), 16), np.int32)
    cta_st = np.zeros(int(info[1]) + 1, np.int32)
    _check(lib().bsp_spmm_plan_inspect(*args, _ptr(units), _ptr(cta), _ptr(steps), _ptr(stages),
                                       _ptr(cta_st)))
    keys = ["units", "ctas", "group_rows", "n_tiles", "slab", "kc", "stages", "steps",
            "plan_bytes", "smem_bytes", "tmem_cols", "variant", "producers", "stage_list", "nsub",
            "step_stride"]
    d = {k: int(info[i]) for i, k in enumerate(keys)}
    d.update(unit_table=units, cta_begin=cta, step_table=steps[: int(info[7])],
             stage_table=stages[: int(info[13])], cta_stage_begin=cta_st)
    # row-stacked plans: stacking order of the block-rows (None = consecutive)
    d["entry_rows"] = None
    if d["variant"] == 1:
        n = ctypes.c_int64(0)
        eargs = (M, K, R, C, int(rp[-1]), _ptr(rp), _ptr(ci), N, strategy, ctypes.byref(o), sm_count, max_smem)
        _check(lib().bsp_spmm_plan_entry_rows(*eargs, None, ctypes.byref(n)))
        if n.value > 0:
            rows = np.zeros(n.value, np.int32)
            _check(lib().bsp_spmm_plan_entry_rows(*eargs, _ptr(rows), ctypes.byref(n)))
            d["entry_rows"] = rows
    return d


def spmm_plan_traffic(M, K, R, C, row_ptr, col_idx, N, strategy=NAIVE, opts=None, sm_count=148,
                      max_smem=232448):
    """Operand bytes / boxes the SpMM plan moves into shared memory (host only):
    dict(a_bytes, b_bytes, a_boxes, b_boxes, variant)."""
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    ci = np.ascontiguousarray(col_idx, dtype=np.int32)
    ci = ci if ci.size else np.zeros(1, np.int32)
    info = np.zeros(16, np.int64)
    tr = np.zeros(4, np.int64)
    o = opts if opts is not None else Opts()
    _check(lib().bsp_spmm_plan_traffic(M, K, R, C, int(rp[-1]), _ptr(rp), _ptr(ci), N, strategy,
                                       ctypes.byref(o), sm_count, max_smem, _ptr(info), _ptr(tr)))
    return dict(a_bytes=int(tr[0]), b_bytes=int(tr[1]), a_boxes=int(tr[2]), b_boxes=int(tr[3]),
                variant=int(info[11]), units=int(info[0]))


def inspect_sddmm_plan(M, N, R, C, row_ptr, col_idx, K, strategy=NAIVE, opts=None, sm_count=148,
                       max_smem=232448):
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    ci = np.ascontiguousarray(col_idx, dtype=np.int32)
    if ci.size == 0:
        ci = np.zeros(1, np.int32)
    info = np.zeros(16, np.int64)
    o = opts if opts is not None else Opts()
    args = (M, N, R, C, int(rp[-1]), _ptr(rp), _ptr(ci), K, strategy, ctypes.byref(o), sm_count,
            max_smem, _ptr(info))
    _check(lib().bsp_sddmm_plan_inspect(*args, None, None))
    units = np.zeros((max(int(info[0]), 1), int(info[12])), np.int32)
    cta = np.zeros(int(info[1]) + 1, np.int32)
    _check(lib().bsp_sddmm_plan_inspect(*args, _ptr(units), _ptr(cta)))
    return dict(units=int(info[0]), ctas=int(info[1]), slab=int(info[4]), kc=int(info[5]),
                stages=int(info[6]), keep_a=int(info[7]), variant=int(info[11]), nseg_max=int(info[13]),
                producers=int(info[14]), unit_table=units[: int(info[0])], cta_begin=cta)


def ipc_export(dev: Device, tensor):
    """(64-byte handle, byte offset) that lets another process on this node map
    the device allocation holding `tensor`."""
    h = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    off = ctypes.c_int64()
    _check(lib().bsp_ipc_export(dev.handle, _ptr(tensor), h, ctypes.byref(off)))
    return h.raw, int(off.value)


def ipc_import(dev: Device, handle: bytes) -> int:
    """Map a peer process's allocation into this one; returns its base address."""
    base = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(bytes(handle), IPC_HANDLE_BYTES)
    _check(lib().bsp_ipc_import(dev.handle, buf, ctypes.byref(base)))
    return int(base.value)


def ipc_close(dev: Device, base: int) -> None:
    _check(lib().bsp_ipc_close(dev.handle, ctypes.c_void_p(base)))


def partition_rows(row_ptr: np.ndarray, parts: int) -> np.ndarray:
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    bounds = np.zeros(parts + 1, dtype=np.int64)
    _check(lib().bsp_partition_rows(_ptr(rp), rp.size - 1, parts, _ptr(bounds)))
    return bounds


def serpentine_assign(n: int, parts: int):
    owner = np.zeros(max(n, 1), dtype=np.int32)
    slot = np.zeros(max(n, 1), dtype=np.int32)
    _check(lib().bsp_serpentine_assign(n, parts, _ptr(owner), _ptr(slot)))
    return owner[:n], slot[:n]
