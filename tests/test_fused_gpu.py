"""Fused decoder-layer kernels against the stock transformers modules they
replace in the decode rounds' forwards (Qwen3RMSNorm, q_norm / k_norm +
apply_rotary_pos_emb + the cache append, Qwen3MLP's act_fn(gate) * up).

float32: max |out - ref| <= 1e-5 * max |ref| (the reduction order of the
mean differs).  bf16: the same rounding steps as the stock modules, so at
least 99% of elements are identical and none differs by more than 2 bf16
ulps of the reference's magnitude."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _k():
    from ddtree_eagle3_patch_b200 import kernels
    return kernels


def _close(out, ref, dtype):
    out, ref = out.float(), ref.float()
    if dtype == torch.float32:
        assert (out - ref).abs().max() <= 1e-5 * ref.abs().max(), (out - ref).abs().max()
    else:
        same = (out == ref).float().mean().item()
        assert same >= 0.99, same
        ulp = 2.0 ** -7
        assert ((out - ref).abs() <= 2 * ulp * ref.abs().clamp_min(1e-3)).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,cols", [(33, 2560), (16, 4096), (1, 96), (5, 1000)])
def test_rms_norm_matches_qwen3_rmsnorm(dtype, rows, cols):
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm
    g = torch.Generator(device=DEV).manual_seed(rows * cols)
    x = (3 * torch.randn(rows, cols, generator=g, device=DEV)).to(dtype)
    norm = Qwen3RMSNorm(cols, eps=1e-6).to(DEV, dtype)
    with torch.no_grad():
        norm.weight.copy_((1 + 0.2 * torch.randn(cols, generator=g, device=DEV)).to(dtype))
        ref = norm(x)
    _close(_k().rms_norm(x, norm.weight, 1e-6), ref, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("ctx", [0, 5])
def test_qk_norm_rope_append_matches_stock_ops(dtype, ctx):
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm, apply_rotary_pos_emb
    K = _k()
    hq, hkv, T, cap = 32, 8, 33, 300
    g = torch.Generator(device=DEV).manual_seed(11 + ctx)
    q_raw = torch.randn(T, hq * 128, generator=g, device=DEV).to(dtype)
    k_new = torch.randn(T, hkv * 128, generator=g, device=DEV).to(dtype)
    v_new = torch.randn(T, hkv * 128, generator=g, device=DEV).to(dtype)
    k_ctx = torch.randn(max(ctx, 1), hkv * 128, generator=g, device=DEV).to(dtype)[:ctx]
    v_ctx = torch.randn(max(ctx, 1), hkv * 128, generator=g, device=DEV).to(dtype)[:ctx]
    qn, kn = Qwen3RMSNorm(128, 1e-6).to(DEV, dtype), Qwen3RMSNorm(128, 1e-6).to(DEV, dtype)
    with torch.no_grad():
        qn.weight.copy_((1 + 0.1 * torch.randn(128, generator=g, device=DEV)).to(dtype))
        kn.weight.copy_((1 + 0.1 * torch.randn(128, generator=g, device=DEV)).to(dtype))
    pos = torch.arange(ctx + T, device=DEV).float() + 97.0
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, device=DEV).float() / 128))
    emb = torch.cat([pos[:, None] * inv, pos[:, None] * inv], -1)
    cos, sin = emb.cos().to(dtype), emb.sin().to(dtype)
    cache_k = torch.zeros(1, hkv, cap, 128, dtype=dtype, device=DEV)
    cache_v = torch.zeros_like(cache_k)
    start, ctx_off, ctx_cnt = 200, 190, max(ctx - 2, 0)
    rs = torch.tensor([start, ctx_off, ctx_cnt, 0], dtype=torch.int32, device=DEV)
    q_out = K.qk_norm_rope_append(q_raw, k_new, v_new, qn.weight, kn.weight, 1e-6, 1e-6, cos, sin, cache_k,
                                  cache_v, rs, hq, hkv, ctx_k=k_ctx if ctx else None, ctx_v=v_ctx if ctx else None)
    with torch.no_grad():
        kv_k = torch.cat([k_ctx, k_new]) if ctx else k_new
        kv_v = torch.cat([v_ctx, v_new]) if ctx else v_new
        q = qn(q_raw.view(1, T, hq, 128)).transpose(1, 2)
        k = kn(kv_k.view(1, ctx + T, hkv, 128)).transpose(1, 2)
        c, s = cos[None], sin[None]
        q_ref, _ = apply_rotary_pos_emb(q, q, c[:, -T:], s[:, -T:])
        k_ref, _ = apply_rotary_pos_emb(k, k, c, s)
    _close(q_out, q_ref[0].transpose(0, 1), dtype)
    exp_k = torch.zeros_like(cache_k)
    exp_v = torch.zeros_like(cache_v)
    exp_k[:, :, start: start + T] = k_ref[:, :, ctx:]
    exp_v[:, :, start: start + T] = v_new.view(T, hkv, 128).transpose(0, 1)[None]
    if ctx_cnt:
        exp_k[:, :, ctx_off: ctx_off + ctx_cnt] = k_ref[:, :, :ctx_cnt]
        exp_v[:, :, ctx_off: ctx_off + ctx_cnt] = v_ctx[:ctx_cnt].view(ctx_cnt, hkv, 128).transpose(0, 1)[None]
    _close(cache_k, exp_k, dtype)
    assert torch.equal(cache_v, exp_v)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_silu_mul_matches_act_times_up(dtype):
    from transformers.activations import ACT2FN
    g = torch.Generator(device=DEV).manual_seed(5)
    gate = (4 * torch.randn(33, 9728, generator=g, device=DEV)).to(dtype)
    up = torch.randn(33, 9728, generator=g, device=DEV).to(dtype)
    ref = ACT2FN["silu"](gate) * up
    _close(_k().silu_mul(gate, up), ref, dtype)
