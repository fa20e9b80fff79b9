"""Error behaviour of the C ABI (the reference's boundary returns an error code
and launches nothing on bad input: gpu-d1/src/learn.cu:643-708). Every call
here is rejected by argument checks that run before any CUDA call, so the test
needs no GPU: a null or misaligned pointer, a size out of range or a layout
the kernels do not support returns D1_ERR_BAD_ARGUMENT, and empty batches
return 0 where the header documents it."""
import ctypes as C

import pytest

BAD = 9002


@pytest.fixture(scope='module')
def lib():
    from d1 import _lib
    return _lib.library()


FAKE = 1 << 20          # a 16-byte-aligned address that is never dereferenced
MIS = FAKE + 2          # a misaligned one


def test_gemm_rejects_bad_shapes_and_layouts(lib):
    g = lambda **kw: lib.d1_gemm(kw.get('a', FAKE), kw.get('lda', 64), kw.get('b', FAKE), kw.get('ldb', 64),
                                 kw.get('M', 128), kw.get('N', 256), kw.get('K', 64), None, 0, None, 0,
                                 kw.get('c', FAKE), kw.get('ldc', 256), None, 0, kw.get('cf'), kw.get('ldcf', 0),
                                 kw.get('splits', 1), None)
    assert g(M=0) == BAD and g(N=0) == BAD and g(K=0) == BAD
    assert g(a=MIS) == BAD and g(b=MIS) == BAD and g(c=MIS) == BAD
    assert g(lda=60) == BAD                      # pitch below K
    assert g(lda=68) == BAD                      # pitch not a multiple of 16 bytes
    assert g(ldc=100) == BAD                     # output pitch below N
    assert g(splits=0) == BAD
    assert g(splits=2, K=1024, lda=1024, ldb=1024) == BAD   # split-K writes fp32 slabs only
    assert g(c=None) == BAD                      # no output at all
    assert lib.d1_gemm_splits(0, 4) == BAD and lib.d1_gemm_splits(1832, 64) == 29
    # the same rules for the pair kernel and the general form
    p = lambda **kw: lib.d1_gemm_pair(FAKE, kw.get('lda', 2048), 0, FAKE, 2048, 0, kw.get('M', 65536), 256, 2048,
                                      None, 0, None, 0, FAKE, 256, None, 0, kw.get('splits', 1), None)
    assert p(M=0) == BAD and p(lda=2044) == BAD and p(splits=0) == BAD
    # compact-operand forms: aligned compact rows, B of the 1832-feature width,
    # an expanded B no wider than the 1840-column [X | 1] layout
    ca = lambda **kw: lib.d1_gemm_cobs_a(kw.get('cobs', FAKE), None, kw.get('M', 1024), FAKE, 1832, 256, None, 0,
                                         FAKE, 256, None)
    assert ca(M=0) == BAD and ca(cobs=MIS) == BAD and ca(cobs=None) == BAD
    cb = lambda **kw: lib.d1_gemm_cobs_b(FAKE, 256, kw.get('cobs', FAKE), FAKE, 256, kw.get('N', 1840), 4096, FAKE,
                                         1840, 8, None)
    assert cb(N=1848) == BAD and cb(cobs=MIS) == BAD and cb(N=0) == BAD


def test_env_and_head_entry_points(lib):
    # spec env: negative batch, missing config
    assert lib.d1_spec_step(FAKE, -1, None, FAKE, FAKE, FAKE, FAKE, None, None) == BAD
    assert lib.d1_spec_crop(FAKE, 4, 8, FAKE, None) == BAD      # D4 element out of range
    assert lib.d1_spec_crop(FAKE, 0, 0, FAKE, None) == 0         # empty batch
    # policy head: only the 256-wide hidden layer exists
    assert lib.d1_policy_head_sample(FAKE, 8, 128, FAKE, FAKE, None, 0, 0, 0, FAKE, None, None, None, None) == BAD
    assert lib.d1_policy_head_sample(FAKE, 0, 256, FAKE, FAKE, None, 0, 0, 0, FAKE, None, None, None, None) == 0
    assert lib.d1_ar_head_sample(FAKE, -1, FAKE, FAKE, FAKE, FAKE, 0, 0, 0, None, None, None, None, None, None,
                                 None, None) == BAD
    # D4 camera transform: 16-byte aligned rows
    assert lib.d1_spec_d4_observe(MIS, FAKE, FAKE, 4, FAKE, FAKE, None) == BAD
    assert lib.d1_spec_d4_observe(FAKE, FAKE, FAKE, 0, FAKE, FAKE, None) == 0
    assert lib.d1_spec_d4_draw(FAKE, 4, FAKE, 1, None, 0, 0, 0, None) == BAD   # outcome rows narrower than 2
    # conv layers: 1..3 only
    assert lib.d1_conv_layer(4, FAKE, 1, FAKE, FAKE, FAKE, None) == BAD
    assert lib.d1_conv_layer(1, MIS, 1, FAKE, FAKE, FAKE, None) == BAD


def test_ppo_entry_points(lib):
    from d1.ppo import GradJob
    assert lib.d1_ppo_gather_x(FAKE, 1830, FAKE, 16, FAKE, 1840, 1, None) == BAD   # F not a multiple of 8
    assert lib.d1_ppo_gather_x(FAKE, 1832, FAKE, 16, FAKE, 1832, 1, None) == BAD   # no room for the ones column
    jobs = (GradJob * 5)()
    assert lib.d1_grad_reduce(jobs, 5, None) == BAD                                # more than 4 jobs
    bad = (GradJob * 1)(GradJob(FAKE, 100, 1, 1, 100, 120, 1, FAKE, None))         # cols_out > cols_in
    assert lib.d1_grad_reduce(bad, 1, None) == BAD
    short = (GradJob * 1)(GradJob(FAKE, 50, 2, 1, 100, 100, 1, FAKE, None))        # partials overlap
    assert lib.d1_grad_reduce(short, 1, None) == BAD
    ok_job = (GradJob * 1)(GradJob(FAKE, 128, 2, 1, 128, 128, 1, FAKE, None))
    ptrs = (C.c_void_p * 9)(*([FAKE] * 9))
    # peer exchange: 2..8 ranks, a rank inside the world, the stride holds the gradient
    step = lambda world, rank, stride: lib.d1_ppo_step_peer(ok_job, 1, FAKE, FAKE, FAKE, FAKE, 128, 1e-3, 0.9,
                                                            0.999, 1e-5, 0.5, FAKE, None, 0, ptrs, ptrs, stride,
                                                            world, rank, 0, None)
    assert step(9, 0, 128) == BAD and step(1, 0, 128) == BAD and step(2, 2, 128) == BAD
    assert step(2, 0, 126) == BAD
    assert lib.d1_peer_alloc(0, C.byref(C.c_void_p()), (C.c_char * 64)()) == BAD
