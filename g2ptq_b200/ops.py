"""Torch-tensor wrappers over the C ABI (include/g2ptq_b200.h).

Every function takes CUDA tensors, checks devices / dtypes / contiguity, pulls
the current CUDA stream, allocates any workspace through the torch caching
allocator and calls the library.  No function here computes anything itself.
"""

import ctypes
import os

import torch

from . import _lib
from ._lib import call, query

_DT = {torch.bfloat16: _lib.DTYPE_BF16, torch.float32: _lib.DTYPE_F32,
       torch.float16: _lib.DTYPE_F16}


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _cuda(*tensors):
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("g2ptq_b200 ops require CUDA tensors (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("g2ptq_b200 ops require every tensor on the same device")
    return dev


def _contig(*tensors):
    for t in tensors:
        if t is not None and not t.is_contiguous():
            raise ValueError("g2ptq_b200 ops require contiguous tensors")


def dtype_code(dtype):
    try:
        return _DT[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}")


def workspace(nbytes, device):
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


_DEVICE_STATUS = {}


def device_status(device):
    """The status word (device int32 [1]) that tensor-core launches without a
    caller-given one report to: G2Q_ERR_TIMEOUT when a pipeline wait gave up.
    ``fasterquant`` reads it with its other status words and raises."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _DEVICE_STATUS.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _DEVICE_STATUS[idx] = t
    return t


def _status(status, device):
    return (device_status(device) if status is None else status).data_ptr()


# --------------------------------------------------------------------------
# Hessian accumulation
# --------------------------------------------------------------------------

def stage_tokens(dst, row0, src, sub=None):
    """Copy ``src`` ([t, C], any row stride) into ``dst[row0:row0+t, :C]``."""
    _cuda(dst, src, sub)
    if src.dim() != 2 or src.stride(1) != 1 or (sub is not None and sub.stride() != src.stride()):
        raise ValueError("stage_tokens expects a 2-D source with unit column stride")
    t, C = src.shape
    call("g2q_stage_tokens", dst.data_ptr(), dtype_code(dst.dtype), dst.stride(0), row0,
         src.data_ptr(), _ptr(sub), dtype_code(src.dtype), src.stride(0), t, C, _stream(dst))


def gram_update(D, A, B=None, row_scale=None, alpha=1.0, beta=1.0, symmetric=None,
                precision=0, status=None):
    """``D <- alpha D + beta A^T diag(s) B`` for token-major ``A [T, M]``, ``B [T, N]``.
    ``status``: device int32 word for a tensor-core timeout (default: the
    device's, ``device_status``)."""
    if B is None:
        B = A
    _cuda(D, A, B, row_scale)
    if symmetric is None:
        symmetric = (B is A) and row_scale is None
    T, M = A.shape
    N = B.shape[1]
    if D.stride(1) != 1 or A.stride(1) != 1 or B.stride(1) != 1:
        raise ValueError("gram_update expects unit column strides")
    ws_bytes = query("g2q_gram_workspace_bytes", M, N, T, precision)
    ws = workspace(ws_bytes, D.device) if ws_bytes else None
    sstride = 0 if row_scale is None else row_scale.stride(0)
    call("g2q_gram_update", D.data_ptr(), D.stride(0), M, N, A.data_ptr(), dtype_code(A.dtype),
         A.stride(0), B.data_ptr(), dtype_code(B.dtype), B.stride(0), _ptr(row_scale), sstride,
         T, int(bool(symmetric)), float(alpha), float(beta), precision, _ptr(ws), ws_bytes,
         _status(status, D.device), _stream(D))


def gram_update_grouped(D, X, scales, alpha=1.0, beta=1.0, precision=0, status=None):
    """``D[g] <- alpha D[g] + beta X^T diag(scales[:, g]) X`` for every row group g:
    ``D [G, C, C]`` contiguous, ``X [T, C]`` token-major, ``scales [T, G]``."""
    _cuda(D, X, scales)
    _contig(D)
    G, C, _ = D.shape
    T = X.shape[0]
    if X.shape[1] != C or X.stride(1) != 1 or scales.shape != (T, G) or scales.stride(1) != 1:
        raise ValueError("gram_update_grouped: shapes or strides do not match")
    if scales.dtype != torch.float32:
        raise TypeError("gram_update_grouped expects fp32 scales")
    ws_bytes = query("g2q_gram_grouped_workspace_bytes", C, T, G, precision)
    ws = workspace(ws_bytes, D.device) if ws_bytes else None
    call("g2q_gram_update_grouped", D.data_ptr(), D.stride(1), D.stride(0), C, X.data_ptr(),
         dtype_code(X.dtype), X.stride(0), scales.data_ptr(), scales.stride(0), G, T,
         float(alpha), float(beta), precision, _ptr(ws), ws_bytes, _status(status, D.device),
         _stream(D))


def sq_colsum(acc, X, keep, scale):
    """``acc <- acc * keep + scale * sum_t X[t]^2``."""
    _cuda(acc, X)
    T, C = X.shape
    call("g2q_sq_colsum", acc.data_ptr(), float(keep), float(scale), X.data_ptr(),
         dtype_code(X.dtype), X.stride(0), T, C, _stream(acc))


# --------------------------------------------------------------------------
# Dense algebra
# --------------------------------------------------------------------------

def gemm(C, A, B, transA=False, transB=False, alpha=0.0, beta=1.0, mask=_lib.MASK_FULL,
         precision=0, status=None):
    """Batched ``C <- alpha C + beta op(A) op(B)`` on fp32 ``[batch, *, *]`` tensors
    (precision 0: fp32 CUDA cores; 1: tensor cores with fp16 hi/lo operands)."""
    _cuda(C, A, B)
    _contig(C, A, B)
    if C.dim() == 2:
        C, A, B = C[None], A[None], B[None]
    batch = C.shape[0]
    M, N = C.shape[1], C.shape[2]
    K = A.shape[1] if transA else A.shape[2]
    sA = A.stride(0) if A.shape[0] > 1 else 0
    sB = B.stride(0) if B.shape[0] > 1 else 0
    if precision == 1:
        nbytes = query("g2q_gemm_tc_workspace_bytes", M, N, K, batch, int(sA != 0), int(sB != 0))
        ws = workspace(nbytes, C.device)
        call("g2q_gemm_tc", C.data_ptr(), C.stride(1), C.stride(0), A.data_ptr(), A.stride(1),
             sA, int(transA), B.data_ptr(), B.stride(1), sB, int(transB), M, N, K, batch,
             float(alpha), float(beta), mask, ws.data_ptr(), nbytes, _status(status, C.device),
             _stream(C))
        return C
    call("g2q_gemm", C.data_ptr(), C.stride(1), C.stride(0), A.data_ptr(), A.stride(1), sA,
         int(transA), B.data_ptr(), B.stride(1), sB, int(transB), M, N, K, batch, float(alpha),
         float(beta), mask, _stream(C))
    return C


# workspace budget of one batched factorization call (bytes)
CHOL_BATCH_BYTES = int(os.environ.get("G2PTQ_B200_CHOL_BATCH_MB", "4096")) << 20


def chol_upper_inverse(H, damp_percent, info=None, precision=0):
    """``U`` with ``U^T U = (H + d I)^-1`` per batch entry; returns ``(U, info)``.

    ``damp_percent`` is a float or a sequence (one per batch entry);
    ``info`` (device int32 [B]) receives 0 / failing pivot / -1 for NaN /
    ``G2Q_ERR_TIMEOUT`` when a tensor-core wait gave up.
    """
    _cuda(H)
    _contig(H)
    Hb = H if H.dim() == 3 else H[None]
    B, C, _ = Hb.shape
    if isinstance(damp_percent, (int, float)):
        damp_percent = [float(damp_percent)] * B
    damps = (_lib.F32 * B)(*[float(d) for d in damp_percent])
    U = torch.empty_like(Hb)
    if info is None:
        info = torch.zeros(B, dtype=torch.int32, device=H.device)
    # precision 1: chains of the batch's factorizations advancing together, as
    # many per chain as CHOL_BATCH_BYTES of workspace holds (at least four);
    # precision 0: up to four side by side on forked streams
    per = query("g2q_chol_workspace_bytes", C)
    chain = min(B, max(4, CHOL_BATCH_BYTES // per)) if precision == 1 else min(B, 4)
    ws_bytes = per * chain + 4096
    ws = workspace(ws_bytes, H.device)
    call("g2q_chol_upper_inverse", U.data_ptr(), Hb.data_ptr(), C, C, B, damps, info.data_ptr(),
         int(precision), ws.data_ptr(), ws_bytes, _stream(H))
    return (U if H.dim() == 3 else U[0]), info


# --------------------------------------------------------------------------
# Quantization
# --------------------------------------------------------------------------

def find_params(scale, zero, W, bits, sym, status=None, param_col=0):
    """Per-row parameters of ``W [rows, cols]`` into column ``param_col`` of
    ``scale`` / ``zero`` ``[rows, ngroups]``."""
    _cuda(scale, zero, W, status)
    rows, cols = W.shape
    if W.stride(1) != 1:
        raise ValueError("find_params expects unit column stride")
    sp = scale[:, param_col] if scale.dim() == 2 else scale
    zp = zero[:, param_col] if zero.dim() == 2 else zero
    pld = scale.stride(0) if scale.dim() == 2 else 1
    call("g2q_find_params", sp.data_ptr(), zp.data_ptr(), pld, W.data_ptr(), rows, cols,
         W.stride(0), bits, int(bool(sym)), _ptr(status), _stream(W))


def find_params_groups(scale, zero, W, bits, sym, groupsize, status=None):
    """``find_params`` of every ``groupsize``-column group of ``W [rows, C]`` in
    one launch, group ``g`` into column ``g`` of ``scale`` / ``zero``."""
    _cuda(scale, zero, W, status)
    rows, C = W.shape
    if W.stride(1) != 1 or scale.stride(1) != 1 or zero.stride() != scale.stride():
        raise ValueError("find_params_groups expects unit column strides")
    count = (C + groupsize - 1) // groupsize
    call("g2q_find_params_groups", scale.data_ptr(), zero.data_ptr(), scale.stride(0),
         W.data_ptr(), rows, C, W.stride(0), bits, int(bool(sym)), 0, count, groupsize,
         _ptr(status), _stream(W))


def clip_config(grid=50, maxshrink=0.5, norm=2.4, hdiag=None, rows_per_block=None):
    """``g2q_clip_t`` for the clip search; ``hdiag [blocks, C]`` (contiguous
    rows) switches to the Hessian-weighted error, each block of
    ``rows_per_block`` weight rows using one row of it."""
    if hdiag is not None:
        _cuda(hdiag)
        if hdiag.dtype != torch.float32 or hdiag.stride(-1) != 1:
            raise ValueError("hdiag must be fp32 with unit column stride")
    return _lib.ClipConfig(int(grid), float(maxshrink), float(norm),
                           None if hdiag is None else hdiag.data_ptr(),
                           0 if hdiag is None else hdiag.stride(0),
                           0 if hdiag is None else int(rows_per_block))


def find_params_clip(scale, zero, W, bits, sym, clip, status=None, param_col=0):
    """``find_params`` with the clip search ``clip`` (a ``clip_config``)."""
    _cuda(scale, zero, W, status)
    rows, cols = W.shape
    if W.stride(1) != 1:
        raise ValueError("find_params expects unit column stride")
    sp = scale[:, param_col] if scale.dim() == 2 else scale
    zp = zero[:, param_col] if zero.dim() == 2 else zero
    pld = scale.stride(0) if scale.dim() == 2 else 1
    call("g2q_find_params_clip", sp.data_ptr(), zp.data_ptr(), pld, W.data_ptr(), rows, cols,
         W.stride(0), bits, int(bool(sym)), ctypes.byref(clip), _ptr(status), _stream(W))


def fake_quantize(W, scale, zero, maxq, colmap=None, out=None, codes=None):
    """Per-element quantize/dequantize of ``W [rows, cols]`` with parameters
    ``scale[r, colmap[c]]`` (``colmap`` None: column 0 of the parameters)."""
    _cuda(W, scale, zero, colmap, out, codes)
    rows, cols = W.shape
    if out is None:
        out = torch.empty(rows, cols, dtype=torch.float32, device=W.device)
    pld = scale.stride(0) if scale.dim() == 2 else 1
    call("g2q_fake_quantize", _ptr(out), 0 if out is None else out.stride(0), _ptr(codes),
         0 if codes is None else codes.stride(0), W.data_ptr(), W.stride(0), rows, cols,
         scale.data_ptr(), zero.data_ptr(), pld, _ptr(colmap), int(maxq), _stream(W))
    return out, codes


def compensate_block(method, W, hinv, scale, zero, colmap, maxq, codes=None, err=None, z=None,
                     ghinv=None, p=None, wraw=None, approx_beta=0.0):
    """One compensation block on ``W [B, rows, ncols]`` (in place -> Q).

    ``err`` (optional) is written column-major ``[B, ncols, rows]`` (the
    reference's kernel layout); ``codes`` is ``[B, rows, ncols]`` int8.
    """
    _cuda(W, hinv, scale, zero, colmap, codes, err, z, ghinv, p, wraw)
    _contig(W, hinv, scale, zero, colmap, codes, err, z, ghinv, p, wraw)
    B, rows, ncols = W.shape
    call("g2q_compensate_block", method, W.data_ptr(), ncols, rows * ncols, B, rows, ncols,
         hinv.data_ptr(), ncols, ncols * ncols, scale.data_ptr(), zero.data_ptr(),
         scale.stride(0) if scale.dim() == 2 else 1, colmap.data_ptr(), int(maxq), _ptr(codes),
         _ptr(err), _ptr(z), _ptr(ghinv), _ptr(p), _ptr(wraw),
         float(approx_beta) if wraw is not None else 0.0, _stream(W))


def compensate(method, W, U, scale, zero, colgroup, dynamic_groups, groupsize, bits, sym,
               blocksize, codes, z=None, gh=None, p=None, status=None, precision=0, clip=None,
               wraw=None, approx_beta=0.0):
    """Whole block traversal (``_run_compensation``); ``W [nl, rows, C]`` -> Q in place.
    ``clip`` (a ``clip_config``) selects the clip search for dynamic groups;
    ``wraw`` / ``approx_beta``: G2PTQ's --approx_grad ablation."""
    _cuda(W, U, scale, zero, colgroup, codes, z, gh, p, status, wraw)
    _contig(W, U, scale, zero, colgroup, codes, z, gh, p, wraw)
    nl, rows, C = W.shape
    ws_bytes = query("g2q_compensate_workspace_bytes", method, nl, rows, C, precision)
    ws = workspace(ws_bytes, W.device)
    call("g2q_compensate", method, W.data_ptr(), nl, rows, C, U.data_ptr(), scale.data_ptr(),
         zero.data_ptr(), scale.shape[1], colgroup.data_ptr(), int(bool(dynamic_groups)),
         int(groupsize), int(bits), int(bool(sym)), int(blocksize), codes.data_ptr(), _ptr(z),
         _ptr(gh), _ptr(p), _ptr(wraw), float(approx_beta) if wraw is not None else 0.0,
         None if clip is None else ctypes.byref(clip), precision,
         ws.data_ptr(), ws_bytes, _ptr(status), _stream(W))


# --------------------------------------------------------------------------
# fasterquant plumbing kernels
# --------------------------------------------------------------------------

def prepare_hessian(H, W=None, extra=None, gzero=None):
    """RTN fallback / dead columns on ``H [nl, C, C]`` (and ``W [nl, rows, C]``)."""
    _cuda(H, W, extra, gzero)
    _contig(H, W, extra, gzero)
    nl, C, _ = H.shape
    rows = 0 if W is None else W.shape[1]
    erows = 0 if extra is None else extra.shape[1]
    if gzero is not None and W is not None and gzero.shape[1] != rows:
        raise ValueError("gzero must have W's layout")
    call("g2q_prepare_hessian", H.data_ptr(), nl, C, _ptr(W), rows, _ptr(extra), erows,
         _ptr(gzero), _stream(H))


def argsort_desc(key):
    _cuda(key)
    perm = torch.empty(key.numel(), dtype=torch.int64, device=key.device)
    call("g2q_argsort_desc", perm.data_ptr(), key.data_ptr(), key.numel(), _stream(key))
    return perm


def mean_diag(H):
    _cuda(H)
    _contig(H)
    nl, C, _ = H.shape
    key = torch.empty(C, dtype=torch.float32, device=H.device)
    call("g2q_mean_diag", key.data_ptr(), H.data_ptr(), nl, C, _stream(H))
    return key


def permute_cols(src, perm, inverse=False, out=None):
    _cuda(src, perm, out)
    _contig(src, perm)
    x = src if src.dim() == 3 else src[None]
    if out is None:
        out = torch.empty_like(src)
    call("g2q_permute_cols", out.data_ptr(), src.data_ptr(), src.element_size(), x.shape[0],
         x.shape[1], x.shape[2], perm.data_ptr(), int(inverse), _stream(src))
    return out


def permute_sym(H, perm):
    _cuda(H, perm)
    _contig(H)
    out = torch.empty_like(H)
    nl, C, _ = H.shape
    call("g2q_permute_sym", out.data_ptr(), H.data_ptr(), nl, C, perm.data_ptr(), _stream(H))
    return out


def cast_check(src, dtype, nan_count, out=None):
    _cuda(src, nan_count)
    _contig(src)
    if out is None:
        out = torch.empty(src.shape, dtype=dtype, device=src.device)
    call("g2q_cast_check", out.data_ptr(), dtype_code(dtype), src.data_ptr(), src.numel(),
         nan_count.data_ptr(), _stream(src))
    return out


def pack_upper(H, scale=1.0, out=None):
    """Upper triangles of ``H [B, C, C]`` (or ``[C, C]``) packed row by row,
    times ``scale`` -> fp32 ``[B * C(C+1)/2]`` (``out`` may be a view of a
    larger buffer)."""
    _cuda(H, out)
    Hb = H if H.dim() == 3 else H[None]
    B, C, _ = Hb.shape
    if Hb.stride(2) != 1 or (B > 1 and Hb.stride(0) < C * Hb.stride(1)):
        raise ValueError("pack_upper expects unit column stride")
    n = B * C * (C + 1) // 2
    if out is None:
        out = torch.empty(n, dtype=torch.float32, device=H.device)
    if out.numel() != n or not out.is_contiguous():
        raise ValueError("pack_upper: out must be contiguous with B * C(C+1)/2 elements")
    call("g2q_pack_upper", out.data_ptr(), Hb.data_ptr(), C, Hb.stride(1), Hb.stride(0), B,
         float(scale), _stream(H))
    return out


def unpack_upper(H, packed, mirror=True):
    """Fill ``H [B, C, C]`` (or ``[C, C]``) from ``pack_upper``'s layout: the
    lower triangle mirrored, or zero (``mirror=False``, a triangular factor)."""
    _cuda(H, packed)
    Hb = H if H.dim() == 3 else H[None]
    B, C, _ = Hb.shape
    if packed.numel() != B * C * (C + 1) // 2 or not packed.is_contiguous():
        raise ValueError("unpack_upper: packed has the wrong size")
    call("g2q_unpack_upper", Hb.data_ptr(), packed.data_ptr(), C, Hb.stride(1), Hb.stride(0), B,
         int(bool(mirror)), _stream(H))
    return H


def pack_int32(codes, bits):
    _cuda(codes)
    _contig(codes)
    rows, cols = codes.shape
    factor = 32 // bits
    out = torch.empty(rows, -(-cols // factor), dtype=torch.int32, device=codes.device)
    call("g2q_pack_int32", out.data_ptr(), codes.data_ptr(), rows, cols, bits, _stream(codes))
    return out


def trust_region_beta(grad, GH, Qsub, Wsub, dinv, alpha):
    _cuda(grad, GH, Qsub, Wsub, dinv)
    _contig(grad, GH, Qsub, Wsub, dinv)
    nl, rows, C = grad.shape
    beta = torch.empty(nl, rows, dtype=torch.float32, device=grad.device)
    call("g2q_trust_region_beta", beta.data_ptr(), grad.data_ptr(), GH.data_ptr(),
         Qsub.data_ptr(), Wsub.data_ptr(), dinv.data_ptr(), nl, rows, C, float(alpha),
         _stream(grad))
    return beta


def diag_of_utu(U):
    _cuda(U)
    _contig(U)
    nl, C, _ = U.shape
    out = torch.empty(nl, C, dtype=torch.float32, device=U.device)
    call("g2q_diag_of_utu", out.data_ptr(), U.data_ptr(), nl, C, _stream(U))
    return out


def scale_rows(X, s):
    _cuda(X, s)
    _contig(X, s)
    nl, rows, C = X.shape
    call("g2q_scale_rows", X.data_ptr(), s.data_ptr(), nl, rows, C, _stream(X))
    return X


# --------------------------------------------------------------------------
# G2PTQ refresh step: saliency / gradient caches and the block-loss heads
# --------------------------------------------------------------------------

def _rows2d(t):
    """``t`` viewed as ``[rows, t.shape[-1]]`` with unit column stride."""
    t2 = t.reshape(-1, t.shape[-1]) if t.dim() != 2 else t
    if t2.shape[-1] > 1 and t2.stride(-1) != 1:
        t2 = t2.contiguous()
    return t2


def saliency(grad, num_groups, out=None):
    """``[T, G]`` fp32 group means of ``grad**2`` over ``grad``'s last dim."""
    _cuda(grad, out)
    g2 = _rows2d(grad)
    T, R = g2.shape
    if R % num_groups:
        raise RuntimeError(f"shape '[{T}, {num_groups}, {R / num_groups}]' is invalid for "
                           f"input of size {T * R}")
    if out is None:
        out = torch.empty(T, num_groups, dtype=torch.float32, device=grad.device)
    _contig(out)
    call("g2q_saliency", out.data_ptr(), g2.data_ptr(), dtype_code(g2.dtype),
         g2.stride(0) if T > 1 else R, T, R, int(num_groups), _stream(g2))
    return out


def scaled_accumulate(out, x, w, first):
    """``out <- (0 if first else out) + w * x`` (fp32, same shapes)."""
    _cuda(out, x)
    _contig(out, x)
    if out.dtype != torch.float32 or x.dtype != torch.float32 or out.numel() != x.numel():
        raise ValueError("scaled_accumulate takes two fp32 tensors of the same size")
    call("g2q_scaled_accumulate", out.data_ptr(), x.data_ptr(), out.numel(), float(w),
         int(bool(first)), _stream(out))
    return out


def running_mean(cache, grad, keep, inv, first):
    """``cache <- (0 if first else cache * keep) + grad * inv`` (cache fp32)."""
    _cuda(cache, grad)
    _contig(cache, grad)
    if cache.dtype != torch.float32 or cache.numel() != grad.numel():
        raise ValueError("running_mean takes an fp32 cache of the gradient's size")
    call("g2q_running_mean", cache.data_ptr(), grad.data_ptr(), dtype_code(grad.dtype),
         grad.numel(), float(keep), float(inv), int(bool(first)), _stream(cache))
    return cache


def block_loss_forward(kind, x, target=None, labels=None):
    """Block-loss head over the rows of ``x`` (last dim = V).  Returns
    ``(loss, row_stats, x2, t2, labels)``: an fp32 scalar, the per-row
    statistics the backward needs and the 2-D operands it reads."""
    _cuda(x, target, labels)
    x2 = _rows2d(x)
    rows, V = x2.shape
    t2 = None
    if kind == _lib.LOSS_NLL:
        labels = labels.reshape(-1)
        if labels.dtype != torch.int64 or labels.numel() != rows:
            raise ValueError("labels must be int64 with one entry per row")
        labels = labels.contiguous()
    else:
        if target is None or target.shape != x.shape:
            raise ValueError("target must have the shape of x")
        if target.dtype != x.dtype:
            raise TypeError("target and x must have the same dtype")
        t2 = _rows2d(target)
    loss = torch.empty((), dtype=torch.float32, device=x.device)
    stats = torch.empty(max(rows, 1), 3, dtype=torch.float32, device=x.device)
    call("g2q_block_loss_forward", int(kind), loss.data_ptr(), stats.data_ptr(), x2.data_ptr(),
         _ptr(t2), _ptr(labels), dtype_code(x2.dtype), x2.stride(0) if rows > 1 else V,
         (t2.stride(0) if rows > 1 else V) if t2 is not None else V, rows, V, _stream(x2))
    return loss, stats, x2, t2, labels


def block_loss_backward(kind, stats, x2, t2, labels, grad_scale=None):
    """Gradient of the block loss with respect to the 2-D ``x2`` (same dtype),
    times the fp32 scalar tensor ``grad_scale`` (None = 1)."""
    rows, V = x2.shape
    grad = torch.empty(rows, V, dtype=x2.dtype, device=x2.device)
    gs = None
    if grad_scale is not None:
        gs = grad_scale.reshape(()).to(torch.float32).contiguous()
    call("g2q_block_loss_backward", int(kind), grad.data_ptr(), V, stats.data_ptr(),
         x2.data_ptr(), _ptr(t2), _ptr(labels), dtype_code(x2.dtype),
         x2.stride(0) if rows > 1 else V,
         (t2.stride(0) if rows > 1 else V) if t2 is not None else V, _ptr(gs), rows, V,
         _stream(x2))
    return grad
