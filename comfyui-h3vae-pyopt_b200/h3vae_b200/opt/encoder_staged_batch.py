"""Staged clip batching of a klvae-shaped encoder (mirror of the reference's
opt/encoder_staged_batch.py): the first `cut` down stages (the prefix) run per 17-frame clip, the
rest (the suffix) on batches of up to `batch_size` clips, and the clip latents are concatenated in
time.  Clips stay independent: batching only stacks them along the batch axis.  This build's own
runtime does the same with its INT8 encoder (runtime.H3VAEPyOptRuntime.encode); these classes serve
a caller that holds a klvae encoder module."""
from __future__ import annotations

import torch
import torch.nn.functional as F

_CL3 = torch.channels_last_3d
_SUPPORTED = ((1, 1), (1, 2), (2, 1), (2, 2), (2, 4))


def _run_stages(h, stages):
    for stage in stages:
        for block in stage.block:
            h = block(h)
        if hasattr(stage, "downsample"):
            h = stage.downsample(h)
    return h


class EncoderPrefix(torch.nn.Module):
    """conv_in and the first `cut` down stages.  ref: opt/encoder_staged_batch.py:6-21."""

    def __init__(self, encoder, cut):
        super().__init__()
        if cut not in (1, 2):
            raise ValueError("Only validated split locations 1 and 2 supported")
        if encoder.gradient_checkpointing or encoder.use_fused_norm:
            raise ValueError("Expected inference encoder without fused-norm flag")
        self.conv_in = encoder.conv_in
        self.stages = torch.nn.ModuleList(list(encoder.down[:cut]))

    def forward(self, x):
        return _run_stages(self.conv_in(x.contiguous(memory_format=_CL3)), self.stages)


class EncoderSuffix(torch.nn.Module):
    """The remaining down stages, norm_out -> SiLU -> conv_out, and the quant conv.
    ref: opt/encoder_staged_batch.py:24-36."""

    def __init__(self, encoder, quant_conv, cut):
        super().__init__()
        self.stages = torch.nn.ModuleList(list(encoder.down[cut:]))
        self.norm_out = encoder.norm_out
        self.conv_out = encoder.conv_out
        self.quant_conv = quant_conv

    def forward(self, h):
        h = _run_stages(h, self.stages)
        return self.quant_conv(self.conv_out(F.silu(self.norm_out(h))))


def encode_staged(normalized_video, prefix, suffix, *, clip_length, token_drop, batch_size, cut):
    """[1, C, T, H, W] normalized video -> moments concatenated over clips; T is padded to a multiple
    of clip_length by repeating the last frame and the last token_drop latent frames are dropped.
    ref: opt/encoder_staged_batch.py:39-57."""
    if normalized_video.ndim != 5 or normalized_video.shape[0] != 1:
        raise ValueError("Expected batch-one video")
    if (cut, batch_size) not in _SUPPORTED:
        raise ValueError("Unsupported combination; avoid large int32-indexed tensors")
    x = normalized_video
    pad = (-x.shape[2]) % clip_length
    if pad:
        x = torch.cat([x, x[:, :, -1:].expand(-1, -1, pad, -1, -1)], dim=2)
    x = x.contiguous(memory_format=_CL3)
    starts = list(range(0, x.shape[2], clip_length))
    outputs = []
    for g in range(0, len(starts), batch_size):
        group = starts[g:g + batch_size]
        features = [prefix(x[:, :, t:t + clip_length]) for t in group]
        batch = torch.cat(features, dim=0).contiguous(memory_format=_CL3)
        moments = suffix(batch)
        outputs.extend(moments[i:i + 1] for i in range(len(group)))
        del features, batch, moments
    out = torch.cat(outputs, dim=2)
    return out[:, :, :-token_drop] if token_drop else out


__all__ = ["EncoderPrefix", "EncoderSuffix", "encode_staged"]
