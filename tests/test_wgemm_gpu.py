"""The weight-streaming tcgen05 GEMM (ddt_wgemm) against a float32 reference
of the same bf16 inputs, at the projection shapes of the Qwen3-4B verify and
draft forwards and at edge sizes.

Tolerance: bf16 output of an fp32-accumulated product, |y - ref| <=
1e-2 * max |ref|; split-K sums in a fixed order, so two runs are identical."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _k():
    from ddtree_eagle3_patch_b200 import kernels
    return kernels


def _case(T, N, K, seed, residual=False, x_pad=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    xs = torch.randn(T, K + x_pad, generator=g, device=DEV).to(torch.bfloat16)
    x = xs[:, :K]
    w = (torch.randn(N, K, generator=g, device=DEV) / K ** 0.5).to(torch.bfloat16)
    r = torch.randn(T, N, generator=g, device=DEV).to(torch.bfloat16) if residual else None
    ref = x.float() @ w.float().T
    if r is not None:
        ref = ref + r.float()
    return x, w, r, ref


@pytest.mark.parametrize("T,N,K", [
    (33, 2560, 4096),     # o_proj (split K)
    (33, 2560, 9728),     # down_proj (split K)
    (33, 6144, 2560),     # packed q/k/v
    (33, 19456, 2560),    # packed gate/up
    (16, 2560, 2560),     # draft rows
    (15, 151936, 2560),   # draft lm_head
    (1, 128, 64),
    (64, 384, 640),
    (48, 256, 128),
    (17, 1024, 4096),
    (65, 2560, 4096),     # budget-64 verify rows (token tile 80)
    (65, 19456, 2560),
    (100, 384, 640),      # token tile 128
    (128, 256, 512),
])
def test_wgemm_matches_float32(T, N, K):
    x, w, _, ref = _case(T, N, K, seed=T * 7 + N)
    y = _k().wgemm(x, w)
    torch.cuda.synchronize()
    assert _k().wgemm_status(DEV) == 0
    err = (y.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item(), err
    assert torch.equal(y, _k().wgemm(x, w))          # split-K order is fixed


@pytest.mark.parametrize("T,N,K", [(33, 2560, 4096), (33, 2560, 9728), (16, 256, 512), (65, 2560, 9728),
                                   (128, 2560, 4096)])
def test_wgemm_residual_and_strided_rows(T, N, K):
    x, w, r, ref = _case(T, N, K, seed=N + K, residual=True, x_pad=64)
    assert x.stride(0) == K + 64
    y = _k().wgemm(x, w, residual=r)
    err = (y.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item(), err
    # the addmm it replaces, within the same tolerance
    torch_y = torch.addmm(r, x, w.T)
    assert (y.float() - torch_y.float()).abs().max().item() <= 1e-2 * ref.abs().max().item()


def test_wgemm_rejects_unsupported_shapes():
    K = _k()
    x = torch.zeros(129, 128, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(128, 128, dtype=torch.bfloat16, device=DEV)
    assert not K.wgemm_supported(x, w)
    assert not K.wgemm_supported(x[:4], torch.zeros(100, 128, dtype=torch.bfloat16, device=DEV))
    with pytest.raises(ValueError):
        K.wgemm(x, w)


@pytest.mark.parametrize("T,I,K,splits", [
    (33, 9728, 2560, 1),    # Qwen3-4B MLP, one CTA per 128 packed rows
    (33, 9728, 2560, 2),    # the same through the cluster reduction
    (16, 9728, 2560, 0),    # draft rows, automatic split
    (5, 128, 256, 4),
    (64, 256, 512, 0),
    (65, 9728, 2560, 1),    # budget-64 verify rows, token tile 80
    (65, 9728, 2560, 2),
    (128, 512, 1024, 3),    # token tile 128 through the cluster reduction
])
def test_wgemm_gate_up_equals_separate_products(T, I, K, splits):
    """The fused epilogue rounds gate and up to bf16, then SiLU, then the
    product: bit-equal to two plain launches with the same split count
    followed by the elementwise kernel, and within bf16 rounding of the
    float32 product."""
    kern = _k()
    g = torch.Generator(device=DEV).manual_seed(T + I + splits)
    x = torch.randn(T, K, generator=g, device=DEV).to(torch.bfloat16)
    wg = (torch.randn(I, K, generator=g, device=DEV) / K ** 0.5).to(torch.bfloat16)
    wu = (torch.randn(I, K, generator=g, device=DEV) / K ** 0.5).to(torch.bfloat16)
    wp = kern.interleave_gate_up(wg, wu)
    assert torch.equal(wp[64:128], wu[:64]) and torch.equal(wp[128:192], wg[64:128])
    s = splits if splits else 0
    y = kern.wgemm_gate_up(x, wp, splits=s)
    torch.cuda.synchronize()
    assert kern.wgemm_status(DEV) == 0
    if s:
        sep = kern.silu_mul(kern.wgemm(x, wg, splits=s), kern.wgemm(x, wu, splits=s))
        assert torch.equal(y, sep)
    gate = (x.float() @ wg.float().T).to(torch.bfloat16)
    up = (x.float() @ wu.float().T).to(torch.bfloat16)
    ref = (torch.nn.functional.silu(gate) * up).float()
    err = (y.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item(), err
    assert torch.equal(y, kern.wgemm_gate_up(x, wp, splits=s))


def _layer_chain(kern, x, w_norm, wo, wp, wd):
    """rms_norm -> projection with residual -> rms_norm -> gate/up -> down
    with residual: every launch reads the one before it."""
    h = kern.rms_norm(x, w_norm, 1e-6)
    x2 = kern.wgemm(h, wo, residual=x)
    h2 = kern.rms_norm(x2, w_norm, 1e-6)
    a = kern.wgemm_gate_up(h2, wp)
    return kern.wgemm(a, wd, residual=x2)


def test_pdl_chain_matches_serial_eager_and_graph():
    """Launched as programmatic dependents, a chain of dependent kernels
    gives the bit-identical result of the serialised launches, eagerly and
    replayed from a CUDA graph (each kernel waits for its predecessor before
    touching its output; only weights load early)."""
    kern = _k()
    g = torch.Generator(device=DEV).manual_seed(5)
    H, I, T = 2560, 9728, 33
    x = torch.randn(T, H, generator=g, device=DEV).to(torch.bfloat16)
    w_norm = (1 + 0.1 * torch.randn(H, generator=g, device=DEV)).to(torch.bfloat16)
    wo = (torch.randn(H, H, generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
    wp = (torch.randn(2 * I, H, generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
    wd = (torch.randn(H, I, generator=g, device=DEV) / I ** 0.5).to(torch.bfloat16)
    ref = _layer_chain(kern, x, w_norm, wo, wp, wd)
    for _ in range(3):
        ref = _layer_chain(kern, ref, w_norm, wo, wp, wd)
    torch.cuda.synchronize()
    with kern.pdl():
        y = x
        for _ in range(4):
            y = _layer_chain(kern, y, w_norm, wo, wp, wd)
        torch.cuda.synchronize()
        assert torch.equal(y, ref)
        xin = x.clone()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            gy = xin
            for _ in range(4):
                gy = _layer_chain(kern, gy, w_norm, wo, wp, wd)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(gy, ref)
    assert kern.wgemm_status(DEV) == 0
    del graph


def test_pdl_attention_reads_rows_written_just_before():
    """The draft layout under PDL: the launch before the attention appends
    context rows below the prefix length and the block rows at it; with
    stable_dev at the context offset the attention equals the serialised
    run (keys the append writes never load early)."""
    kern = _k()
    g = torch.Generator(device=DEV).manual_seed(9)
    hq, hkv, cap, n = 32, 8, 1024, 16
    k_cache = torch.randn(hkv, cap, 128, generator=g, device=DEV).to(torch.bfloat16)
    v_cache = torch.randn(hkv, cap, 128, generator=g, device=DEV).to(torch.bfloat16)
    start, ctx = 700, 300
    rs = torch.tensor([start, start - ctx, ctx], dtype=torch.int32, device=DEV)
    q = torch.randn(n, hq, 128, generator=g, device=DEV).to(torch.bfloat16)
    k_new = torch.randn(hkv, ctx + n, 128, generator=g, device=DEV).to(torch.bfloat16)
    v_new = torch.randn(hkv, ctx + n, 128, generator=g, device=DEV).to(torch.bfloat16)
    bits = torch.full((n, 1), -1, dtype=torch.int32, device=DEV)
    ws = kern.attention_workspace(n, hq, hkv, cap - n, DEV)

    def run(kc, vc):
        kern.kv_append(k_new[:, :ctx], v_new[:, :ctx], kc, vc, rs[1:2])
        kern.kv_append(k_new[:, ctx:], v_new[:, ctx:], kc, vc, rs[0:1])
        return kern.tree_attention(q, kc, vc, cap - n, bits, 0.088, past_dev=rs[0:1], workspace=ws,
                                   stable_dev=rs[1:2])

    kc0, vc0 = k_cache.clone(), v_cache.clone()
    ref = run(kc0, vc0)
    torch.cuda.synchronize()
    with kern.pdl():
        out = run(k_cache.clone(), v_cache.clone())
        torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert kern.attention_status(DEV, ws) == 0
