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
])
def test_wgemm_matches_float32(T, N, K):
    x, w, _, ref = _case(T, N, K, seed=T * 7 + N)
    y = _k().wgemm(x, w)
    torch.cuda.synchronize()
    assert _k().wgemm_status(DEV) == 0
    err = (y.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item(), err
    assert torch.equal(y, _k().wgemm(x, w))          # split-K order is fixed


@pytest.mark.parametrize("T,N,K", [(33, 2560, 4096), (33, 2560, 9728), (16, 256, 512)])
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
    x = torch.zeros(65, 128, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(128, 128, dtype=torch.bfloat16, device=DEV)
    assert not K.wgemm_supported(x, w)
    assert not K.wgemm_supported(x[:4], torch.zeros(100, 128, dtype=torch.bfloat16, device=DEV))
    with pytest.raises(ValueError):
        K.wgemm(x, w)
