"""ctypes binding of libspindle_b200.so (the C ABI of include/spindle_gpu.h).

There is no CPU fallback: if the library is missing and cannot be built, or a
call fails, an exception is raised.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("SG_LIB_PATH") or os.path.join(HERE, "libspindle_b200.so")

OK = 0
STATUS = {0: "ok", 1: "invalid argument", 2: "unsupported dtype", 3: "unsupported shape",
          4: "misaligned device pointer", 5: "CUDA error", 6: "NCCL error", 7: "device wait timed out",
          8: "out of memory", 9: "request above the static scratch limit"}


class SgError(RuntimeError):
    def __init__(self, status, what, detail=""):
        self.status = status
        msg = "%s: %s" % (what, STATUS.get(status, "status %d" % status))
        super().__init__(msg + (" (%s)" % detail if detail else ""))


class SgMat(C.Structure):
    _fields_ = [("dtype", C.c_int32), ("layout", C.c_uint32), ("offset", C.c_uint64),
                ("cols", C.c_uint64), ("rows", C.c_uint64)]


class SgQ8K(C.Structure):
    _fields_ = [("d", C.c_void_p), ("qs", C.c_void_p), ("bsums", C.c_void_p), ("n", C.c_uint64)]


MOE_MAX_USED = 16


class SgMoeChoice(C.Structure):
    _fields_ = [("n", C.c_uint32), ("pad_", C.c_uint32 * 3), ("id", C.c_int32 * MOE_MAX_USED),
                ("weight", C.c_float * MOE_MAX_USED)]


class SgMoe(C.Structure):
    _fields_ = [("router", C.c_void_p), ("gate_up", C.c_void_p), ("down", C.c_void_p),
                ("gate_up_dtype", C.c_int32), ("down_dtype", C.c_int32),
                ("gate_up_stride", C.c_uint64), ("down_stride", C.c_uint64),
                ("dim", C.c_uint64), ("n_ff", C.c_uint64), ("n_expert", C.c_uint64), ("n_used", C.c_uint64),
                ("norm", C.c_int32), ("moe_prune", C.c_float),
                ("shared_gate_up", C.c_void_p), ("shared_down", C.c_void_p),
                ("shared_gate_up_dtype", C.c_int32), ("shared_down_dtype", C.c_int32),
                ("shared_n_ff", C.c_uint64), ("shared_gate", C.c_void_p)]


TP_MAX_RANKS = 8


class SgTpGroup(C.Structure):
    _fields_ = [("n_ranks", C.c_uint32), ("rank", C.c_uint32), ("recv", C.c_void_p * TP_MAX_RANKS),
                ("comm", C.c_void_p)]


class SgMoeEp(C.Structure):
    _fields_ = [("n_ranks", C.c_uint32), ("rank", C.c_uint32), ("expert_lo", C.c_uint64), ("expert_hi", C.c_uint64),
                ("recv_slots", C.c_uint64), ("recv", C.c_void_p * TP_MAX_RANKS), ("comm", C.c_void_p)]


P, U64, I32 = C.c_void_p, C.c_uint64, C.c_int32

# name -> (restype, argtypes); every function the header declares.
SIGNATURES = {
    "sg_status_string": (C.c_char_p, [I32]),
    "sg_last_error_string": (C.c_char_p, []),
    "sg_row_bytes": (I32, [I32, U64, C.POINTER(U64)]),
    "sg_supports": (I32, [C.POINTER(SgMat)]),
    "sg_set_int_kernels": (None, [I32]),
    "sg_int_kernels_enabled": (I32, []),
    "sg_q8k_bytes": (U64, [U64]),
    "sg_q8k_view": (I32, [P, U64, C.POINTER(SgQ8K)]),
    "sg_alloc": (I32, [U64, C.POINTER(P)]),
    "sg_free": (I32, [P]),
    "sg_upload": (I32, [P, U64, C.POINTER(P)]),
    "sg_memcpy_h2d": (I32, [P, P, U64, P]),
    "sg_memcpy_d2h": (I32, [P, P, U64, P]),
    "sg_stream_sync": (I32, [P]),
    "sg_device_status": (I32, []),
    "sg_q8k_quantize": (I32, [P, U64, U64, U64, C.POINTER(SgQ8K), P]),
    "sg_matmul_rows": (I32, [P, C.POINTER(SgMat), C.POINTER(SgQ8K), C.POINTER(P), U64, U64, U64, P]),
    "sg_matvec": (I32, [P, C.POINTER(SgMat), P, U64, P, U64, U64, U64, U64, P]),
    "sg_matvec_list": (I32, [C.POINTER(P), C.POINTER(SgMat), C.POINTER(P), C.POINTER(P), U64, P]),
    "sg_matvec_list_q8k": (I32, [C.POINTER(P), C.POINTER(SgMat), C.POINTER(P), C.POINTER(P), U64, P]),
    "sg_q8k_image_bytes": (U64, [U64]),
    "sg_q8k_images": (I32, [C.POINTER(P), C.POINTER(U64), C.POINTER(P), U64, P]),
    "sg_matvec_rows_float": (I32, [P, C.POINTER(SgMat), P, U64, P, U64, U64, U64, U64, P]),
    "sg_matmul_batch_scratch_bytes": (U64, [C.POINTER(SgMat), U64]),
    "sg_matmul_batch": (I32, [P, C.POINTER(SgMat), P, U64, P, U64, U64, U64, U64, P, U64, P]),
    "sg_matmul_rows_float": (I32, [P, C.POINTER(SgMat), P, U64, P, U64, U64, U64, U64, P]),
    "sg_ipc_handle_bytes": (U64, []),
    "sg_ipc_get_handle": (I32, [P, P]),
    "sg_ipc_open": (I32, [P, C.POINTER(P)]),
    "sg_ipc_close": (I32, [P]),
    "sg_tp_comm_bytes": (U64, []),
    "sg_tp_comm_init": (I32, [P, P]),
    "sg_tp_recv_bytes": (U64, [U64, U64]),
    "sg_matvec_tp": (I32, [P, C.POINTER(SgMat), P, U64, U64, U64, U64, P, U64, P, P]),
    "sg_matvec_scratch_bytes": (U64, [U64, U64]),
    "sg_matvec_scratch": (I32, [P, C.POINTER(SgMat), P, U64, P, U64, U64, U64, U64, P, U64, P]),
    "sg_matvec_static": (I32, [P, C.POINTER(SgMat), P, U64, P, U64, U64, U64, U64, P]),
    "sg_block_sums": (I32, [P, C.POINTER(SgMat), C.POINTER(SgQ8K), P, U64, U64, P]),
    "sg_libm_eval": (I32, [I32, U64, U64, U64, P, P]),
    "sg_binary_version": (I32, [P]),
    "sg_q4k_gemv_4row": (I32, [P, U64, P, P, U64, P, P]),
    "sg_q4k_gemm_spec4": (I32, [P, U64, U64, P, P, U64, P]),
    "sg_route_moe_top2": (I32, [P, P, U64, P, P, P]),
    "sg_flash_gqa_spec4": (I32, [P, P, P, P, P, U64, U64, P]),
    "sg_quantize_weights": (I32, [I32, P, U64, U64, P, P]),
    "sg_tiled16_bytes": (I32, [I32, U64, U64, C.POINTER(U64)]),
    "sg_repack_tiled16": (I32, [I32, P, U64, U64, P, P]),
    "sg_unpack_tiled16": (I32, [I32, P, U64, U64, P, P]),
    "sg_moe_pack_gate_up": (I32, [I32, P, P, U64, U64, U64, P, P]),
    "sg_moe_pack_down": (I32, [I32, P, U64, U64, U64, P, P]),
    "sg_moe_scratch_bytes": (U64, [C.POINTER(SgMoe)]),
    "sg_moe_forward": (I32, [C.POINTER(SgMoe), P, P, P, U64, P, P, P]),
    "sg_moe_batch_scratch_bytes": (U64, [C.POINTER(SgMoe), U64]),
    "sg_moe_forward_batch": (I32, [C.POINTER(SgMoe), P, U64, U64, P, U64, P, U64, P, P]),
    "sg_moe_ep_recv_bytes": (U64, [C.POINTER(SgMoe), U64]),
    "sg_moe_forward_batch_ep": (I32, [C.POINTER(SgMoe), C.POINTER(SgMoeEp), P, U64, U64, P, U64, P, U64, P, P]),
    "sg_model_scratch_bytes": (U64, [P]),
    "sg_model_kv_bytes": (U64, [P]),
    "sg_model_prepare": (I32, [P, P, U64, P]),
    "sg_forward": (I32, [P, P, P, P, U64, P, P, P, P]),
    "sg_model_ep_scratch_bytes": (U64, [P]),
    "sg_kv_shift": (I32, [P, P, P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, P]),
    "sg_forward_ep": (I32, [P, P, P, P, P, U64, P, P, P, P]),
    "sg_forward_batch_range": (I32, [P, C.c_uint32, C.c_uint32, P, P, U64, P, P, P, U64, U64, P, P, U64, P, P]),
    "sg_pipe_recv_bytes": (U64, [U64]),
    "sg_pipe_send": (I32, [P, U64, U64, P, P, P]),
    "sg_pipe_recv": (I32, [P, U64, U64, P, P, P, P]),
    "sg_model_batch_scratch_bytes": (U64, [P, U64]),
    "sg_model_batch_prepare": (I32, [P, U64, P, U64, P]),
    "sg_forward_batch": (I32, [P, P, U64, P, P, P, U64, U64, P, U64, P, P]),
}

_lib = None


def load(build_if_missing=True):
    """Loads the library, building it first when it is missing or stale and
    nvcc is available (the GPU box ships the prebuilt .so)."""
    global _lib
    if _lib is not None:
        return _lib
    try:
        from . import build as _build
        if os.path.exists(_build.NVCC) and build_if_missing and not os.environ.get("SG_LIB_PATH"):
            _build.build()
    except Exception:
        if not os.path.exists(LIB_PATH):
            raise
    if not os.path.exists(LIB_PATH):
        raise RuntimeError("libspindle_b200.so is missing; run spindle_b200/build.py")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        f = getattr(lib, name)
        f.restype, f.argtypes = res, args
    _lib = lib
    return lib


def check(status, what):
    if status != OK:
        detail = ""
        if status == 5 and _lib is not None:
            detail = _lib.sg_last_error_string().decode(errors="replace")
        raise SgError(status, what, detail)
