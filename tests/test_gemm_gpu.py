"""tcgen05 GEMM against a PyTorch fp32 restatement of the same op (bf16 inputs,
fp32 accumulation): relative error bound 2e-3 on bf16 outputs, 1e-4 on fp32."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def G():
    from d1 import gemm
    return gemm


def ref(a, b, bias=None, relu=False):
    y = a.float() @ b.float().T
    if bias is not None:
        y = y + bias
    return y.relu() if relu else y


@pytest.mark.parametrize('M,N,K', [(128, 256, 64), (65536, 256, 1832), (4096, 256, 256), (1000, 256, 1832),
                                   (16384, 13, 256), (300, 1832, 256)])
def test_bf16_out_with_bias_relu(G, M, N, K):
    g = torch.Generator(device='cuda').manual_seed(M + N + K)
    a = torch.randn(M, K, device='cuda', generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device='cuda', generator=g) / K ** 0.5).to(torch.bfloat16)
    bias = torch.randn(N, device='cuda', generator=g)
    ldc = (N + 7) // 8 * 8
    out = torch.empty((M, ldc), dtype=torch.bfloat16, device='cuda')[:, :N]
    G.gemm(a, b, bias=bias, relu=True, out=out)
    torch.cuda.synchronize()
    assert G.gemm_error() == 0
    r = ref(a, b, bias, True)
    err = (out.float() - r).abs().max().item()
    assert err <= 2e-3 * r.abs().max().item() + 1e-2, err


def test_transposed_and_fp32_outputs(G):
    M, N, K = 2048, 256, 512
    a = torch.randn(M, K, device='cuda').to(torch.bfloat16)
    b = torch.randn(N, K, device='cuda').to(torch.bfloat16)
    ct = torch.empty((N, M), dtype=torch.bfloat16, device='cuda')
    cf = torch.empty((1, M, N), device='cuda')
    G.gemm(a, b, out_t=ct, out_f32=cf)
    r = ref(a, b)
    assert torch.allclose(cf[0], r, rtol=1e-4, atol=1e-3)
    assert torch.allclose(ct.float(), r.T, rtol=1e-2, atol=1e-1)


def test_split_k_partials_sum_to_the_product(G):
    M, N, K = 256, 1832, 16384
    a = torch.randn(M, K, device='cuda').to(torch.bfloat16)
    b = torch.randn(N, K, device='cuda').to(torch.bfloat16)
    s = G.splits_for(K, 16)
    ld = (N + 3) // 4 * 4
    cf = torch.empty((s, M, ld), device='cuda')
    G.gemm(a, b, out_f32=cf[:, :, :N], splits=16)
    r = ref(a, b)
    got = cf[:, :, :N].sum(0)
    assert torch.allclose(got, r, rtol=1e-4, atol=1e-2)


@pytest.mark.parametrize('M,N,K,splits', [(128, 256, 64, 1), (256, 1832, 16384, 8), (300, 200, 640, 1), (256, 1832, 4096, 4)])
def test_b_stored_k_by_n(G, M, N, K, splits):
    """d1_gemm_bkn: B given as [K, N] (MN-major operand) -- bf16 out and split-K
    fp32 slabs against the fp32 product."""
    g = torch.Generator(device='cuda').manual_seed(M + N + K)
    a = (torch.randn(M, K, device='cuda', generator=g) / K ** 0.5).to(torch.bfloat16)
    b = torch.randn(K, N, device='cuda', generator=g).to(torch.bfloat16)
    ref = a.float() @ b.float()
    ld = (N + 7) // 8 * 8
    if splits == 1:
        bias = torch.randn(N, device='cuda', generator=g)
        out = torch.empty((M, ld), dtype=torch.bfloat16, device='cuda')[:, :N]
        G.gemm_bkn(a, b, bias=bias, relu=True, out=out)
        want = torch.relu(ref + bias)
        assert torch.allclose(out.float(), want, rtol=2e-2, atol=2e-2 * want.abs().max().item())
    used = G.splits_for(K, splits)
    slabs = torch.empty((used, M, ld), device='cuda')
    G.gemm_bkn(a, b, out_f32=slabs[:, :, :N], splits=splits)
    got = slabs[:, :, :N].sum(0)
    assert torch.allclose(got, ref, rtol=1e-3, atol=1e-3 * ref.abs().max().item())
    assert G.gemm_error() == 0


@pytest.mark.parametrize('M,N,K,splits', [(256, 256, 16384, 64), (256, 1832, 16384, 8), (192, 100, 320, 1)])
def test_both_operands_stored_k_major_rows(G, M, N, K, splits):
    """d1_gemm_ex with A stored [K, M] and B stored [K, N] (both MN-major
    operands): the weight-gradient shape dW = dY^T X of the PPO backward."""
    g = torch.Generator(device='cuda').manual_seed(M * 7 + N + K)
    ld = (N + 7) // 8 * 8  # TMA row pitches are multiples of 16 bytes
    lm = (M + 7) // 8 * 8
    a_km = (torch.randn(K, lm, device='cuda', generator=g) / K ** 0.5).to(torch.bfloat16)[:, :M]
    b_kn = torch.randn(K, ld, device='cuda', generator=g).to(torch.bfloat16)[:, :N]
    ref = a_km.float().T @ b_kn.float()
    used = G.splits_for(K, splits)
    slabs = torch.empty((used, M, ld), device='cuda')
    G.gemm_ex(a_km, b_kn, a_kn=True, b_kn=True, out_f32=slabs[:, :, :N], splits=splits)
    got = slabs[:, :, :N].sum(0)
    assert torch.allclose(got, ref, rtol=1e-3, atol=1e-3 * ref.abs().max().item())
    if splits == 1:
        out = torch.empty((M, ld), dtype=torch.bfloat16, device='cuda')[:, :N]
        G.gemm_ex(a_km, b_kn, a_kn=True, b_kn=True, out=out)
        assert torch.allclose(out.float(), ref, rtol=2e-2, atol=2e-2 * ref.abs().max().item())
    assert G.gemm_error() == 0


def test_gathered_rows_match_the_gathered_copy(G):
    """d1_gemm_rows: A rows and MN-major B K-rows taken from a table through an
    index array (TMA tile::gather4) equal the product over the explicit gather
    -- the PPO's layer 1 and dW1 on a minibatch of the rollout buffer."""
    g = torch.Generator(device='cuda').manual_seed(5)
    rows, F, mb = 40000, 1832, 4096
    table = (torch.randn(rows, F, device='cuda', generator=g) / F ** 0.5).to(torch.bfloat16)
    idx = torch.randperm(rows, device='cuda', generator=g)[:mb]
    x = table[idx]
    w = torch.randn(256, F, device='cuda', generator=g).to(torch.bfloat16)
    b = torch.randn(256, device='cuda', generator=g)
    h_ref = torch.empty((mb, 256), dtype=torch.bfloat16, device='cuda')
    G.gemm(x, w, bias=b, relu=True, out=h_ref)
    h = G.gemm_rows(table, w, a_rows=idx, bias=b, relu=True)
    assert torch.equal(h, h_ref)
    dy = torch.randn(mb, 256, device='cuda', generator=g).to(torch.bfloat16)
    used = G.splits_for(mb, 8)
    s_ref = torch.empty((used, 256, F), device='cuda')
    s = torch.empty((used, 256, F), device='cuda')
    G.gemm_ex(dy, x, a_kn=True, b_kn=True, out_f32=s_ref, splits=8)
    G.gemm_rows(dy, table, b_rows=idx, a_kn=True, b_kn=True, out_f32=s, splits=8)
    assert torch.equal(s, s_ref)
    # M tail: 1000 rows
    h2 = G.gemm_rows(table, w, a_rows=idx[:1000], bias=b, relu=True)
    assert torch.equal(h2, h_ref[:1000])
    assert G.gemm_error() == 0


@pytest.mark.parametrize('M,N,K,a_kn,b_kn,splits', [(65536, 256, 1832, False, False, 1), (1000, 256, 1832, False, False, 1),
                                                     (128, 13, 256, False, False, 1), (300, 1832, 256, False, False, 1),
                                                     (4096, 256, 4096, True, True, 8), (256, 1832, 8192, True, True, 16),
                                                     (8192, 256, 256, False, True, 1), (2048, 512, 1024, True, False, 4),
                                                     (40000, 256, 640, False, False, 1), (38000, 384, 512, True, True, 1)])
def test_pair_kernel_matches_the_product(G, M, N, K, a_kn, b_kn, splits):
    """2-SM pair kernel: K-major and MN-major operands, ragged M and N, split-K
    slabs, 256- and 512-row pair tiles (65,536, 40,000 and 38,000 rows take the
    latter); bf16 output with bias + ReLU + mask, and fp32 slabs equal to the
    one-CTA kernel's."""
    g = torch.Generator(device='cuda').manual_seed(M + 3 * N + K)
    a = torch.randn(M, K, device='cuda', generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device='cuda', generator=g) / K ** 0.5).to(torch.bfloat16)
    pad = lambda t: torch.nn.functional.pad(t, (0, (-t.shape[1]) % 8)).contiguous()[:, :t.shape[1]]
    aa = pad(a.T.contiguous()) if a_kn else a
    bb = pad(b.T.contiguous()) if b_kn else b
    r = ref(a, b)
    ld = (N + 7) // 8 * 8
    s = G.splits_for(K, splits)
    cf = torch.empty((s, M, ld), device='cuda')
    G.gemm_pair(aa, bb, a_kn, b_kn, out_f32=cf[:, :, :N], splits=splits)
    one = torch.empty((s, M, ld), device='cuda')
    G.gemm_ex(aa, bb, a_kn, b_kn, out_f32=one[:, :, :N], splits=splits, single=True)
    torch.cuda.synchronize()
    assert G.gemm_error() == 0
    assert torch.allclose(cf[:, :, :N].sum(0), r, rtol=1e-3, atol=1e-2)
    assert torch.equal(cf[:, :, :N], one[:, :, :N])
    if splits == 1:
        bias = torch.randn(N, device='cuda', generator=g)
        mask = pad(torch.randn(M, N, device='cuda', generator=g).to(torch.bfloat16))
        out = torch.empty((M, ld), dtype=torch.bfloat16, device='cuda')[:, :N]
        G.gemm_pair(aa, bb, a_kn, b_kn, bias=bias, relu=True, mask=mask, out=out)
        want = torch.empty((M, ld), dtype=torch.bfloat16, device='cuda')[:, :N]
        G.gemm_ex(aa, bb, a_kn, b_kn, bias=bias, relu=True, mask=mask, out=want, single=True)
        torch.cuda.synchronize()
        assert G.gemm_error() == 0
        assert torch.equal(out, want)
        rr = torch.where(mask.float() > 0, ref(a, b, bias, True), 0.)
        assert (out.float() - rr).abs().max().item() <= 2e-3 * rr.abs().max().item() + 1e-2


@pytest.mark.parametrize('M', [16384, 65536, 3000])
def test_compact_operand_products_equal_the_expanded_products(G, M):
    """Products with one operand expanded from compact observation rows inside
    the pair kernel (four expander warps writing the swizzled tile) equal the
    same products on the explicitly expanded one-hot matrix bit for bit: the
    layer-1 forward (A expanded, gathered rows; 512-row pair tiles at 65,536)
    and the weight + bias gradient (B expanded, with the ones column)."""
    from d1._lib import library
    lib = library()
    g = torch.Generator(device='cuda').manual_seed(M)
    rows = M + 777
    cobs = torch.zeros((rows, 320), dtype=torch.uint8, device='cuda')
    cobs[:, :225] = torch.randint(0, 8, (rows, 225), device='cuda', generator=g, dtype=torch.uint8)
    cobs[:, 256:].view(torch.bfloat16).copy_(torch.randn(rows, 32, device='cuda', generator=g))
    idx = torch.randperm(rows, device='cuda', generator=g)[:M]
    x = torch.empty((M, 1840), dtype=torch.bfloat16, device='cuda')
    assert lib.d1_ppo_gather_cobs(cobs.data_ptr(), idx.data_ptr(), M, x.data_ptr(), 1840, 1,
                                  torch.cuda.current_stream().cuda_stream) == 0
    w = (torch.randn(256, 1832, device='cuda', generator=g) / 40).to(torch.bfloat16)
    bias = torch.randn(256, device='cuda', generator=g)
    got = G.gemm_cobs_a(cobs, w, idx=idx, bias=bias, relu=True)
    want = G.gemm_ex(x[:, :1832], w, bias=bias, relu=True)
    torch.cuda.synchronize()
    assert G.gemm_error() == 0
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    # weight gradient: A = dh [K = M samples, 256], B = X [K, 1840]
    dh = (torch.randn(M, 256, device='cuda', generator=g)).to(torch.bfloat16)
    s = G.splits_for(M, 8)
    got_s = torch.empty((s, 256, 1840), device='cuda')
    want_s = torch.empty_like(got_s)
    G.gemm_cobs_b(dh, cobs, idx, 1840, got_s, splits=8)
    G.gemm_ex(dh, x, a_kn=True, b_kn=True, out_f32=want_s, splits=8)
    torch.cuda.synchronize()
    assert G.gemm_error() == 0
    assert torch.equal(got_s, want_s)
