"""Vision-tower operators against plain fp32 PyTorch (the reference's own CPU
branches): LayerNorm, GELU-tanh, rotate-half RoPE, Conv3d patch embedding."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _ready():
    from qwen3_5_vl_cuda_custom_b200 import build
    build.build()
    yield
    from qwen3_5_vl_cuda_custom_b200 import kernels as K
    K.device_error_check()


def K():
    from qwen3_5_vl_cuda_custom_b200 import kernels
    return kernels


def close(got, ref, rel=2 ** -7):
    got = got.float().cpu()
    assert (got - ref).abs().max() <= rel * ref.abs().max() + 1e-3, float((got - ref).abs().max())


@pytest.mark.parametrize("rows,cols,with_bias", [(1024, 1152, True), (7, 64, False), (3, 4096, True)])
def test_layernorm(rows, cols, with_bias):
    g = torch.Generator().manual_seed(rows + cols)
    x = (torch.randn(rows, cols, generator=g) * 2 + 0.5).bfloat16()
    w = (1 + 0.1 * torch.randn(cols, generator=g)).bfloat16()
    b = (0.1 * torch.randn(cols, generator=g)).bfloat16() if with_bias else None
    y = K().layernorm(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV), 1e-6)
    ref = F.layer_norm(x.float(), (cols,), w.float(), None if b is None else b.float(), 1e-6)
    close(y, ref)


def test_gelu_tanh():
    g = torch.Generator().manual_seed(1)
    x = (torch.randn(4096, 1152, generator=g) * 3).bfloat16()
    y = K().gelu_tanh(x.to(DEV))
    close(y, F.gelu(x.float(), approximate="tanh"))


def _rope_ref(x, cos, sin):
    dr = cos.shape[-1]
    half = dr // 2
    c = cos.unsqueeze(1) if cos.dim() == 3 else cos[None, None]
    s = sin.unsqueeze(1) if sin.dim() == 3 else sin[None, None]
    x1, x2, xp = x[..., :half], x[..., half:dr], x[..., dr:]
    c1, s1 = c[..., :half], s[..., :half]
    return torch.cat([x1 * c1 - x2 * s1, x2 * c1 + x1 * s1, xp], dim=-1)


@pytest.mark.parametrize("per_batch,dr", [(False, 80), (True, 64), (False, 32)])
def test_rope(per_batch, dr):
    g = torch.Generator().manual_seed(dr)
    B, H, S, D = 2, 16, 100, 80
    x = torch.randn(B, H, S, D, generator=g).bfloat16()
    ang = torch.randn(B if per_batch else 1, S, dr, generator=g)
    cos, sin = ang.cos(), ang.sin()
    if not per_batch:
        cos, sin = cos[0], sin[0]
    y = K().apply_rope(x.to(DEV), cos.to(DEV), sin.to(DEV))
    ref = _rope_ref(x.float(), cos.bfloat16().float(), sin.bfloat16().float())
    close(y, ref)


def test_conv3d_patch():
    g = torch.Generator().manual_seed(3)
    N, C, T, P, E = 1000, 3, 2, 16, 1152
    x = torch.randn(N, C, T, P, P, generator=g).bfloat16()
    w = (torch.randn(E, C, T, P, P, generator=g) * 0.02).bfloat16()
    b = (torch.randn(E, generator=g) * 0.1).bfloat16()
    y = K().conv3d_patch(x.to(DEV), w.to(DEV), b.to(DEV))
    ref = F.conv3d(x.float(), w.float(), b.float(), stride=(T, P, P)).reshape(N, E)
    close(y, ref, rel=1e-2)
