"""Dense layers of the policy on the tcgen05 GEMM (d1_gemm): bf16 in/out, fp32 accumulate."""
import torch

from ._lib import check, library, launch_stream


def _stream(t):
    return launch_stream(t.device)


def gemm(a, b, bias=None, relu=False, out=None, out_t=None, out_f32=None, splits=1, mask=None):
    """act(a @ b.T + bias). a: bf16 [M, K], b: bf16 [N, K] (row pitches may exceed K).
    Any of out (bf16 [M, N]), out_t (bf16 [N, M]) and out_f32 (fp32 [splits, M, N])."""
    M, K = a.shape
    N = b.shape[0]
    assert b.shape[1] == K and a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16
    assert a.stride(1) == 1 and b.stride(1) == 1
    if out is None and out_t is None and out_f32 is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    lib = library()
    check(lib.d1_gemm(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), M, N, K,
                      None if bias is None else bias.data_ptr(), int(relu),
                      None if mask is None else mask.data_ptr(), 0 if mask is None else mask.stride(0),
                      None if out is None else out.data_ptr(), 0 if out is None else out.stride(0),
                      None if out_t is None else out_t.data_ptr(), 0 if out_t is None else out_t.stride(0),
                      None if out_f32 is None else out_f32.data_ptr(), 0 if out_f32 is None else out_f32.stride(-2),
                      splits, _stream(a)), 'd1_gemm')
    return out if out is not None else (out_t if out_t is not None else out_f32)


def splits_for(K, splits):
    return library().d1_gemm_splits(K, splits)


def linear_relu(x, w, b, out=None):
    return gemm(x, w, bias=b, relu=True, out=out)


def gemm_error():
    return library().d1_gemm_error()


def gemm_bkn(a, b_kn, bias=None, relu=False, out=None, out_f32=None, splits=1):
    """act(a @ b_kn + bias) with b_kn stored [K, N] (N contiguous; the tensor-core
    operand is read MN-major). a: bf16 [M, K]. out (bf16 [M, N]) and/or out_f32
    (fp32 [splits, M, N])."""
    M, K = a.shape
    N = b_kn.shape[1]
    assert b_kn.shape[0] == K and a.dtype == torch.bfloat16 and b_kn.dtype == torch.bfloat16
    assert a.stride(1) == 1 and b_kn.stride(1) == 1
    if out is None and out_f32 is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    check(library().d1_gemm_bkn(a.data_ptr(), a.stride(0), b_kn.data_ptr(), b_kn.stride(0), M, N, K,
                                None if bias is None else bias.data_ptr(), int(relu),
                                None if out is None else out.data_ptr(), 0 if out is None else out.stride(0),
                                None if out_f32 is None else out_f32.data_ptr(),
                                0 if out_f32 is None else out_f32.stride(-2), splits, _stream(a)), 'd1_gemm_bkn')
    return out if out is not None else out_f32


def gemm_ex(a, b, a_kn=False, b_kn=False, bias=None, relu=False, out=None, out_t=None, out_f32=None, splits=1,
            mask=None, single=False):
    """act(A @ B^T + bias) with A given as [M, K] (or [K, M] when a_kn) and B as
    [N, K] (or [K, N] when b_kn); the tensor-core operands are then read
    MN-major instead of K-major. Outputs as gemm(). single=True keeps the
    one-CTA kernel for shapes the library would give to the pair kernel."""
    M, K = (a.shape[1], a.shape[0]) if a_kn else a.shape
    N = b.shape[1] if b_kn else b.shape[0]
    assert (b.shape[0] if b_kn else b.shape[1]) == K
    assert a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16 and a.stride(1) == 1 and b.stride(1) == 1
    if out is None and out_t is None and out_f32 is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    p = lambda t: None if t is None else t.data_ptr()
    fn = library().d1_gemm_single if single else library().d1_gemm_ex
    check(fn(a.data_ptr(), a.stride(0), int(a_kn), b.data_ptr(), b.stride(0), int(b_kn), M, N, K, p(bias), int(relu),
             p(mask), 0 if mask is None else mask.stride(0), p(out), 0 if out is None else out.stride(0), p(out_t),
             0 if out_t is None else out_t.stride(0), p(out_f32), 0 if out_f32 is None else out_f32.stride(-2), splits,
             _stream(a)), 'd1_gemm_ex')
    return out if out is not None else (out_t if out_t is not None else out_f32)


def gemm_pair(a, b, a_kn=False, b_kn=False, bias=None, relu=False, out=None, out_f32=None, splits=1, mask=None):
    """gemm_ex on the 2-SM pair kernel (256 x 256 tiles, one per CTA pair)."""
    M, K = (a.shape[1], a.shape[0]) if a_kn else a.shape
    N = b.shape[1] if b_kn else b.shape[0]
    assert (b.shape[0] if b_kn else b.shape[1]) == K
    assert a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16 and a.stride(1) == 1 and b.stride(1) == 1
    if out is None and out_f32 is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    p = lambda t: None if t is None else t.data_ptr()
    check(library().d1_gemm_pair(a.data_ptr(), a.stride(0), int(a_kn), b.data_ptr(), b.stride(0), int(b_kn), M, N, K,
                                 p(bias), int(relu), p(mask), 0 if mask is None else mask.stride(0), p(out),
                                 0 if out is None else out.stride(0), p(out_f32),
                                 0 if out_f32 is None else out_f32.stride(-2), splits, _stream(a)), 'd1_gemm_pair')
    return out if out is not None else out_f32


def gemm_cobs_a(cobs, b, idx=None, M=None, bias=None, relu=False, out=None):
    """act(X . B^T + bias) with X the one-hot expansion of compact observation
    rows cobs[idx] (u8 [rows, 320]; idx int64 [M] or None for the first M rows),
    expanded inside the GEMM; B [N, 1832] bf16."""
    M = idx.shape[0] if idx is not None else (cobs.shape[0] if M is None else M)
    N = b.shape[0]
    assert b.shape[1] == 1832 and b.dtype == torch.bfloat16 and b.stride(1) == 1
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=b.device)
    p = lambda t: None if t is None else t.data_ptr()
    check(library().d1_gemm_cobs_a(cobs.data_ptr(), p(idx), M, b.data_ptr(), b.stride(0), N, p(bias), int(relu),
                                   out.data_ptr(), out.stride(0), _stream(b)), 'd1_gemm_cobs_a')
    return out


def gemm_cobs_b(a_kn, cobs, idx, N, out_f32, splits=1):
    """fp32 split-K slabs of A . X[:, :N] with A given as [K, M] (M contiguous)
    and X the one-hot expansion (+ ones column at 1832) of compact rows
    cobs[idx] (idx int64 [K])."""
    K, M = a_kn.shape
    assert idx.shape[0] == K and a_kn.dtype == torch.bfloat16 and a_kn.stride(1) == 1
    check(library().d1_gemm_cobs_b(a_kn.data_ptr(), a_kn.stride(0), cobs.data_ptr(), idx.data_ptr(), M, N, K,
                                   out_f32.data_ptr(), out_f32.stride(-2), splits, _stream(a_kn)), 'd1_gemm_cobs_b')
    return out_f32


def gemm_rows(a, b, M=None, a_rows=None, b_rows=None, a_kn=False, b_kn=False, bias=None, relu=False, out=None,
              out_f32=None, splits=1, mask=None):
    """gemm_ex with gathered operands: with a_rows (int64 [M]), A's row m is row
    a_rows[m] of the table a [rows, K]; with b_rows (int64 [K], b_kn), B's K-row k
    is row b_rows[k] of the table b [rows, N]."""
    if a_rows is not None:
        M, K = a_rows.shape[0], a.shape[1]
    else:
        M, K = (a.shape[1], a.shape[0]) if a_kn else a.shape
    if b_rows is not None:
        assert b_kn and b_rows.shape[0] == K
        N = b.shape[1]
    else:
        N = b.shape[1] if b_kn else b.shape[0]
    if out is None and out_f32 is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    p = lambda t: None if t is None else t.data_ptr()
    check(library().d1_gemm_rows(a.data_ptr(), a.stride(0), int(a_kn), p(a_rows), a.shape[0] if a_rows is not None else 0,
                                 b.data_ptr(), b.stride(0), int(b_kn), p(b_rows), b.shape[0] if b_rows is not None else 0,
                                 M, N, K, p(bias), int(relu), p(mask), 0 if mask is None else mask.stride(0), p(out),
                                 0 if out is None else out.stride(0), p(out_f32),
                                 0 if out_f32 is None else out_f32.stride(-2), splits, _stream(a)), 'd1_gemm_rows')
    return out if out is not None else out_f32
