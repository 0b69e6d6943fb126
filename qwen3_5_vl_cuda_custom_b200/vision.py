"""Qwen3-VL vision tower on the library's kernels.

Same class names, constructor arguments, parameter names/shapes and forward
signatures as the reference (REF cuda_qwen3_vl/modules/{norms,mlp,attention,
vision_block,vision_patch}.py and models/common.py:25-225), so a reference (or
HF-remapped) state dict loads unchanged:

  CudaVisionTower.forward(hidden_states (seq, C*T*P*P), grid_thw (N, 3))
      -> (pooler_output, last_hidden_state, deepstack_features)

Compute per block: LayerNorm kernel -> fused qkv GEMM (bias in the epilogue)
-> ``q35_vision_qkv_rope_pad`` (split, 2-D rotary in fp32, head-major, head
dim zero-padded to the next size the attention kernels take: 72 -> 128) ->
non-causal tcgen05 attention over the whole sequence (the reference attends
across image boundaries too, REF modules/attention.py:40) -> unpad -> proj
GEMM with bias and the residual add in its epilogue -> LayerNorm -> fc1 (bias)
-> GELU-tanh -> fc2 (bias + residual).  The position-embedding interpolation
and the rotary angle table are index bookkeeping on small tensors, done with
torch ops as in the reference (REF models/common.py:85-174); the embedding
rows are gathered by the row-gather kernel.  bf16 activations; the rotary
angles stay fp32.
"""
from __future__ import annotations

import math

import torch
from torch import nn

from . import _lib
from . import kernels as K
from .configs import VisionConfig
from .modules import CudaEmbedding, CudaLinear


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


class CudaLayerNorm(nn.Module):
    """nn.LayerNorm layout (REF modules/norms.py:25-42)."""

    def __init__(self, dim: int, eps: float = 1e-6, bias: bool = True) -> None:
        super().__init__()
        self.normalized_shape = (dim,)
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))
        if bias:
            self.bias = nn.Parameter(torch.zeros(dim))
        else:
            self.register_parameter("bias", None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return K.layernorm(x, self.weight, self.bias, self.eps)


class CudaVisionMLP(nn.Module):
    """linear_fc1 -> GELU-tanh -> linear_fc2, biases on (REF modules/mlp.py:25-35)."""

    def __init__(self, hidden_size: int, intermediate_size: int) -> None:
        super().__init__()
        self.linear_fc1 = CudaLinear(hidden_size, intermediate_size, bias=True)
        self.linear_fc2 = CudaLinear(intermediate_size, hidden_size, bias=True)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        return self.linear_fc2(K.gelu_tanh(self.linear_fc1(x)), residual=residual)


def _padded_head_dim(D: int) -> int:
    for dp in (32, 64, 128):
        if D <= dp:
            return dp
    raise RuntimeError(f"vision attention: head_dim {D} > 128 is not supported")


class CudaVisionAttention(nn.Module):
    """Non-causal attention with the fused qkv projection and 2-D rotary
    (REF modules/attention.py:11-42).  ``forward(x, cos, sin)`` keeps the
    reference's signature (cos/sin (1, S, D) of the angle table duplicated over
    the two halves); ``forward_angles`` takes the fp32 angle table (S, D/2)."""

    def __init__(self, hidden_size: int, num_heads: int) -> None:
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = hidden_size // num_heads
        self.scale = self.head_dim ** -0.5
        self.qkv = CudaLinear(hidden_size, 3 * hidden_size, bias=True)
        self.proj = CudaLinear(hidden_size, hidden_size, bias=True)

    def forward_angles(self, x: torch.Tensor, angles: torch.Tensor,
                       residual: torch.Tensor | None = None) -> torch.Tensor:
        B, S, C = x.shape
        if B != 1:
            raise RuntimeError("vision attention: batch 1 (the tower flattens images)")
        H, D = self.num_heads, self.head_dim
        Dp = _padded_head_dim(D)
        qkv = self.qkv(x)
        ang = K._require(angles.float(), "vision.angles", torch.float32)
        if ang.shape != (S, D // 2):
            raise RuntimeError(f"vision attention: angles {tuple(ang.shape)}, expected ({S}, {D // 2})")
        q = torch.empty(1, H, S, Dp, device=x.device, dtype=torch.bfloat16)
        k = torch.empty_like(q)
        v = torch.empty_like(q)
        with torch.cuda.device(x.device):
            _lib.call("q35_vision_qkv_rope_pad", qkv.data_ptr(), ang.data_ptr(), q.data_ptr(),
                      k.data_ptr(), v.data_ptr(), S, H, D, Dp, _stream(x))
        out = K.attention_tokens(q, k, v, self.scale, False)  # (1, S, H*Dp)
        if Dp != D:
            o = torch.empty(1, S, H * D, device=x.device, dtype=torch.bfloat16)
            with torch.cuda.device(x.device):
                _lib.call("q35_unpad_heads", out.data_ptr(), o.data_ptr(), S, H, D, Dp, _stream(x))
            out = o
        return self.proj(out, residual=residual)

    def forward(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        # cos/sin carry the angles twice (cat(rot, rot)); recover them once
        ang = torch.atan2(sin.float(), cos.float()).reshape(x.shape[1], -1)[:, : self.head_dim // 2]
        return self.forward_angles(x, ang)


class CudaVisionBlock(nn.Module):
    """x + attn(norm1(x)); x + mlp(norm2(x)) (REF modules/vision_block.py:13-24);
    both residual adds are fused into the projection GEMMs' epilogues."""

    def __init__(self, hidden_size: int, num_heads: int, intermediate_size: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.norm1 = CudaLayerNorm(hidden_size, eps=eps, bias=True)
        self.attn = CudaVisionAttention(hidden_size, num_heads)
        self.norm2 = CudaLayerNorm(hidden_size, eps=eps, bias=True)
        self.mlp = CudaVisionMLP(hidden_size, intermediate_size)

    def forward_angles(self, x: torch.Tensor, angles: torch.Tensor) -> torch.Tensor:
        x = self.attn.forward_angles(self.norm1(x), angles, residual=x)
        return self.mlp(self.norm2(x), residual=x)

    def forward(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        ang = torch.atan2(sin.float(), cos.float()).reshape(x.shape[1], -1)
        return self.forward_angles(x, ang[:, : self.attn.head_dim // 2])


class CudaVisionPatchEmbed(nn.Module):
    """Non-overlapping Conv3d patch embedding as a tcgen05 GEMM
    (REF modules/vision_patch.py:42-63)."""

    def __init__(self, in_channels: int, hidden_size: int, patch_size: int, temporal_patch_size: int) -> None:
        super().__init__()
        self.in_channels = in_channels
        self.hidden_size = hidden_size
        self.patch_size = patch_size
        self.temporal_patch_size = temporal_patch_size
        self.weight = nn.Parameter(torch.empty(hidden_size, in_channels, temporal_patch_size,
                                               patch_size, patch_size))
        self.bias = nn.Parameter(torch.empty(hidden_size))
        nn.init.kaiming_uniform_(self.weight, a=5 ** 0.5)
        nn.init.zeros_(self.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() == 2:
            x = x.view(-1, self.in_channels, self.temporal_patch_size, self.patch_size, self.patch_size)
        return K.conv3d_patch(x, self.weight, self.bias)


class CudaVisionPatchMerger(nn.Module):
    """LayerNorm before (or, with ``use_postshuffle_norm``, after) the
    spatial-merge reshape, then fc1 -> GELU-tanh -> fc2
    (REF modules/vision_patch.py:66-92)."""

    def __init__(self, hidden_size: int, out_hidden_size: int, spatial_merge_size: int = 2,
                 use_postshuffle_norm: bool = False) -> None:
        super().__init__()
        self.hidden_size_in = hidden_size
        self.merged_hidden = hidden_size * (spatial_merge_size ** 2)
        self.use_postshuffle_norm = use_postshuffle_norm
        norm_dim = self.merged_hidden if use_postshuffle_norm else hidden_size
        self.norm = CudaLayerNorm(norm_dim, eps=1e-6, bias=True)
        self.linear_fc1 = CudaLinear(self.merged_hidden, self.merged_hidden, bias=True)
        self.linear_fc2 = CudaLinear(self.merged_hidden, out_hidden_size, bias=True)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.use_postshuffle_norm:
            x = self.norm(x.reshape(-1, self.merged_hidden))
        else:
            x = self.norm(x).reshape(-1, self.merged_hidden)
        return self.linear_fc2(K.gelu_tanh(self.linear_fc1(x)))


class _PosEmbedWrap(nn.Module):
    """Keeps the reference's ``pos_embed.emb.weight`` state-dict key."""

    def __init__(self, num_embeddings: int, embedding_dim: int) -> None:
        super().__init__()
        self.emb = CudaEmbedding(num_embeddings, embedding_dim)

    @property
    def weight(self) -> torch.Tensor:
        return self.emb.weight


class CudaVisionTower(nn.Module):
    """Qwen3-VL vision tower (REF models/common.py:25-210)."""

    def __init__(self, cfg: VisionConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.spatial_merge_size = cfg.spatial_merge_size
        self.patch_size = cfg.patch_size
        self.num_grid_per_side = int(math.isqrt(cfg.num_position_embeddings))
        self.patch_embed = CudaVisionPatchEmbed(cfg.in_channels, cfg.hidden_size, cfg.patch_size,
                                                cfg.temporal_patch_size)
        self.pos_embed = _PosEmbedWrap(cfg.num_position_embeddings, cfg.hidden_size)
        head_dim = cfg.hidden_size // cfg.num_heads
        self.head_dim = head_dim
        self.rotary_dim = head_dim // 2
        inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, self.rotary_dim, 2, dtype=torch.float32)
                                             / self.rotary_dim))
        self.register_buffer("inv_freq", inv_freq, persistent=False)
        self.blocks = nn.ModuleList([
            CudaVisionBlock(cfg.hidden_size, cfg.num_heads, cfg.intermediate_size, eps=cfg.rms_norm_eps)
            for _ in range(cfg.num_layers)
        ])
        self.merger = CudaVisionPatchMerger(cfg.hidden_size, cfg.out_hidden_size,
                                            cfg.spatial_merge_size, use_postshuffle_norm=False)
        self.deepstack_mergers = nn.ModuleList([
            CudaVisionPatchMerger(cfg.hidden_size, cfg.out_hidden_size, cfg.spatial_merge_size,
                                  use_postshuffle_norm=True)
            for _ in cfg.deepstack_layers
        ])

    def _apply(self, fn, recurse=True):
        inv = self.inv_freq
        out = super()._apply(fn, recurse)
        if self.inv_freq.dtype != torch.float32:  # rotary math stays fp32
            self.inv_freq = inv.to(device=self.inv_freq.device, dtype=torch.float32)
        return out

    def rotary_angles(self, grid_thw: torch.Tensor) -> torch.Tensor:
        """fp32 (total_tokens, head_dim // 2) angle table: the (row, col) grid
        coordinates in spatial-merge order times inv_freq
        (REF models/common.py:80-120)."""
        m = self.spatial_merge_size
        dev = self.inv_freq.device
        rows = []
        for t, h, w in grid_thw.tolist():
            br = torch.arange(h // m, device=dev)[:, None, None, None] * m
            bc = torch.arange(w // m, device=dev)[None, :, None, None] * m
            ir = torch.arange(m, device=dev)[None, None, :, None]
            ic = torch.arange(m, device=dev)[None, None, None, :]
            r = (br + ir).expand(h // m, w // m, m, m).reshape(-1)
            c = (bc + ic).expand(h // m, w // m, m, m).reshape(-1)
            coords = torch.stack((r, c), dim=-1)
            rows.append(coords.repeat(t, 1) if t > 1 else coords)
        pos = torch.cat(rows).float()  # (total, 2)
        ang = pos[:, :, None] * self.inv_freq[None, None, :]  # (total, 2, rot_half)
        return ang.flatten(1)

    def interpolated_pos_embed(self, grid_thw: torch.Tensor) -> torch.Tensor:
        """Bilinear lookup in the learned position grid, in spatial-merge token
        order (REF models/common.py:122-174); rows gathered by the row-gather
        kernel."""
        m = self.spatial_merge_size
        n = self.num_grid_per_side
        W = self.pos_embed.weight
        dev = W.device
        idx4, w4, sizes = [[], [], [], []], [[], [], [], []], []
        for _t, h, w in grid_thw.tolist():
            hi = torch.linspace(0, n - 1, h)
            wi = torch.linspace(0, n - 1, w)
            hf, wf = hi.int(), wi.int()
            hc, wc = (hf + 1).clip(max=n - 1), (wf + 1).clip(max=n - 1)
            dh, dw = hi - hf, wi - wf
            ids = [(hf[:, None] * n + wf[None]).flatten(), (hf[:, None] * n + wc[None]).flatten(),
                   (hc[:, None] * n + wf[None]).flatten(), (hc[:, None] * n + wc[None]).flatten()]
            ws = [((1 - dh)[:, None] * (1 - dw)[None]).flatten(), ((1 - dh)[:, None] * dw[None]).flatten(),
                  (dh[:, None] * (1 - dw)[None]).flatten(), (dh[:, None] * dw[None]).flatten()]
            for i in range(4):
                idx4[i].append(ids[i])
                w4[i].append(ws[i])
            sizes.append(h * w)
        acc = None
        for i in range(4):
            rows = torch.cat(idx4[i]).to(device=dev, dtype=torch.int32)
            wts = torch.cat(w4[i]).to(device=dev, dtype=torch.float32)
            part = K.gather_rows(W, rows).float() * wts[:, None]
            acc = part if acc is None else acc + part
        out = []
        for emb, (t, h, w) in zip(acc.split(sizes), grid_thw.tolist()):
            emb = emb.repeat(t, 1)
            emb = (emb.view(t, h // m, m, w // m, m, -1).permute(0, 1, 3, 2, 4, 5).flatten(0, 4))
            out.append(emb)
        return torch.cat(out)

    def forward(self, hidden_states: torch.Tensor, grid_thw: torch.Tensor):
        x = self.patch_embed(hidden_states)
        x = (x.float() + self.interpolated_pos_embed(grid_thw)).to(torch.bfloat16)
        ang = self.rotary_angles(grid_thw)
        x = x.unsqueeze(0)
        deep = {layer: i for i, layer in enumerate(self.cfg.deepstack_layers)}
        deepstack_outs = []
        for i, block in enumerate(self.blocks):
            x = block.forward_angles(x, ang)
            if i in deep:
                deepstack_outs.append(self.deepstack_mergers[deep[i]](x.squeeze(0)))
        last = x.squeeze(0)
        return self.merger(last), last, deepstack_outs
