"""ctypes binding of ``libg2ptq_b200.so`` (the C ABI declared in include/g2ptq_b200.h).

The library is built in-tree (``g2ptq_b200/_lib/libg2ptq_b200.so``) by
``g2ptq_b200/build.py``.  There is no fallback: importing an op whose library
is missing raises immediately.
"""

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("G2PTQ_B200_LIB", os.path.join(_HERE, "_lib", "libg2ptq_b200.so"))

ABI_VERSION = 8

G2Q_OK = 0
G2Q_ERR_INVALID_ARG = -1
G2Q_ERR_CUDA = -2
G2Q_ERR_UNSUPPORTED = -3
G2Q_ERR_NONFINITE = -4
G2Q_ERR_TIMEOUT = -5
G2Q_ERR_BAD_SCALE = -6
G2Q_ERR_SCRATCH_LIMIT = -7

DTYPE_BF16, DTYPE_F32, DTYPE_F16 = 0, 1, 2
METHOD_GPTQ, METHOD_G2PTQ, METHOD_GPTAQ = 0, 1, 2
MASK_FULL, MASK_LOWER, MASK_UPPER, MASK_STRICT_UPPER = 0, 1, 2, 3
LOSS_KL, LOSS_NLL, LOSS_MSE = 0, 1, 2

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
F32 = ctypes.c_float
SZ = ctypes.c_size_t


class ClipConfig(ctypes.Structure):
    """``g2q_clip_t``: the clip search of ``find_params`` (--w_clip / --w_hclip)."""
    _fields_ = [("grid", ctypes.c_int), ("maxshrink", ctypes.c_float),
                ("norm", ctypes.c_float), ("hdiag", ctypes.c_void_p),
                ("hdiag_ld", ctypes.c_int64), ("rows_per_block", ctypes.c_int64)]


# name -> argtypes (every entry point returns int unless listed in _RESTYPES)
SIGNATURES = {
    "g2q_abi_version": [],
    "g2q_launch_count": [],
    "g2q_status_string": [I32],
    "g2q_stage_tokens": [P, I32, I64, I64, P, P, I32, I64, I64, I64, P],
    "g2q_set_wait_limit": [I64],
    "g2q_gram_update": [P, I64, I64, I64, P, I32, I64, P, I32, I64, P, I64, I64, I32, F32, F32,
                        I32, P, SZ, P, P],
    "g2q_gram_workspace_bytes": [I64, I64, I64, I32],
    "g2q_gram_update_grouped": [P, I64, I64, I64, P, I32, I64, P, I64, I32, I64, F32, F32, I32, P,
                                SZ, P, P],
    "g2q_gram_grouped_workspace_bytes": [I64, I64, I32, I32],
    "g2q_sq_colsum": [P, F32, F32, P, I32, I64, I64, I64, P],
    "g2q_gemm": [P, I64, I64, P, I64, I64, I32, P, I64, I64, I32, I64, I64, I64, I64, F32, F32,
                 I32, P],
    "g2q_chol_upper_inverse": [P, P, I64, I64, I64, P, P, I32, P, SZ, P],
    "g2q_chol_workspace_bytes": [I64],
    "g2q_find_params": [P, P, I64, P, I64, I64, I64, I32, I32, P, P],
    "g2q_find_params_clip": [P, P, I64, P, I64, I64, I64, I32, I32, P, P, P],
    "g2q_find_params_groups": [P, P, I64, P, I64, I64, I64, I32, I32, I64, I32, I32, P, P],
    "g2q_gemm_tc": [P, I64, I64, P, I64, I64, I32, P, I64, I64, I32, I64, I64, I64, I64, F32, F32,
                    I32, P, SZ, P, P],
    "g2q_gemm_tc_workspace_bytes": [I64, I64, I64, I64, I32, I32],
    "g2q_fake_quantize": [P, I64, P, I64, P, I64, I64, I64, P, P, I64, P, I32, P],
    "g2q_compensate_block": [I32, P, I64, I64, I64, I64, I64, P, I64, I64, P, P, I64, P, I32, P,
                             P, P, P, P, P, F32, P],
    "g2q_compensate": [I32, P, I64, I64, I64, P, P, P, I64, P, I32, I32, I32, I32, I32, P, P, P,
                       P, P, F32, P, I32, P, SZ, P, P],
    "g2q_compensate_workspace_bytes": [I32, I64, I64, I64, I32],
    "g2q_prepare_hessian": [P, I64, I64, P, I64, P, I64, P, P],
    "g2q_argsort_desc": [P, P, I64, P],
    "g2q_mean_diag": [P, P, I64, I64, P],
    "g2q_permute_cols": [P, P, I32, I64, I64, I64, P, I32, P],
    "g2q_permute_sym": [P, P, I64, I64, P, P],
    "g2q_cast_check": [P, I32, P, I64, P, P],
    "g2q_pack_upper": [P, P, I64, I64, I64, I64, F32, P],
    "g2q_unpack_upper": [P, P, I64, I64, I64, I64, I32, P],
    "g2q_pack_int32": [P, P, I64, I64, I32, P],
    "g2q_trust_region_beta": [P, P, P, P, P, P, I64, I64, I64, F32, P],
    "g2q_diag_of_utu": [P, P, I64, I64, P],
    "g2q_scale_rows": [P, P, I64, I64, I64, P],
    "g2q_gram_update_noalloc": [P, I64, I64, I64, P, I32, I64, P, I32, I64, P, I64, I64, I32, F32,
                                F32, P, P],
    "g2q_gram_static_scratch_bytes": [],
    "g2q_saliency": [P, P, I32, I64, I64, I64, I32, P],
    "g2q_scaled_accumulate": [P, P, I64, F32, I32, P],
    "g2q_running_mean": [P, P, I32, I64, F32, F32, I32, P],
    "g2q_block_loss_forward": [I32, P, P, P, P, P, I32, I64, I64, I64, I64, P],
    "g2q_block_loss_backward": [I32, P, I64, P, P, P, P, I32, I64, I64, P, I64, I64, P],
}
_RESTYPES = {
    "g2q_launch_count": ctypes.c_int64,
    "g2q_set_wait_limit": ctypes.c_int64,
    "g2q_status_string": ctypes.c_char_p,
    "g2q_gram_workspace_bytes": SZ,
    "g2q_gram_grouped_workspace_bytes": SZ,
    "g2q_chol_workspace_bytes": SZ,
    "g2q_compensate_workspace_bytes": SZ,
    "g2q_gemm_tc_workspace_bytes": SZ,
    "g2q_gram_static_scratch_bytes": SZ,
}

_lib = None


class G2QError(RuntimeError):
    """A C-ABI call returned a negative status."""

    def __init__(self, name, status):
        self.status = status
        super().__init__(f"{name} failed: {status_string(status)} (status {status})")


def load():
    """Load and bind the library once; raises OSError when it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise OSError(
            f"g2ptq_b200 CUDA library not found at {LIB_PATH}; build it with "
            "`python -m g2ptq_b200.build` (no CPU fallback exists)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = _RESTYPES.get(name, ctypes.c_int)
    got = lib.g2q_abi_version()
    if got != ABI_VERSION:
        raise OSError(f"libg2ptq_b200 ABI {got} does not match the Python binding ({ABI_VERSION})")
    _lib = lib
    return lib


def status_string(status):
    return load().g2q_status_string(int(status)).decode()


def call(name, *args):
    """Invoke an int-returning entry point and raise G2QError on a negative status."""
    fn = getattr(load(), name)
    status = fn(*args)
    if status < 0:
        raise G2QError(name, status)
    return status


def query(name, *args):
    return getattr(load(), name)(*args)
