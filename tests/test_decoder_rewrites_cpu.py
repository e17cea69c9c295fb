"""CPU contracts of the model-rewrite helpers in h3vae_b200.opt (INT8 FFN install, fused FFN,
norm-quant blocks, the norm1 carry chain, INT8 QKV and attention-out projections, QK fusion,
container cloning, the encoder's staged clip batching), following the
reference's tests/test_int8_swiglu_fused.py, test_int8_norm_quant.py, test_int8_qkv.py,
test_int8_attention_out.py and test_kitchen_int8.py:105-127.  The rewritten modules' forward passes
run the ops that the GPU tests cover."""
import copy
from unittest.mock import patch

import pytest
import torch

from h3vae_b200.opt import int8_attention_out, int8_norm_quant, int8_qkv, int8_swiglu_fused, kitchen_int8
from h3vae_b200.opt._containers import clone_containers, selected_indices


def _attn_block(width=2048):
    block = torch.nn.Module()
    block.attn = torch.nn.Module()
    block.attn.original = torch.nn.Module()
    block.attn.original.to_qkv = torch.nn.Linear(width, width * 3, device="meta")
    block.attn.original.to_out = torch.nn.Linear(width, width, device="meta")
    return block.eval()


def _int8both_ff():
    ff = torch.nn.Module()
    ff.mode = "INT8both"
    ff.w1 = torch.nn.Linear(4, 8)
    ff.w2 = torch.nn.Linear(4, 4)
    return ff


def test_selected_indices():
    """ref: tests/test_int8_qkv.py:10-14."""
    assert selected_indices(36) == tuple(range(36))
    assert selected_indices(36, [3, 7]) == (3, 7)
    for bad in ([], [1, 1], [-1], [36], [True], [1.0]):
        with pytest.raises(ValueError):
            selected_indices(36, bad)


def test_fused_ffn_requires_quantized_ffn_and_clone_isolates():
    """ref: tests/test_int8_swiglu_fused.py:20-40."""
    with pytest.raises(ValueError):
        int8_swiglu_fused.FusedFFN(torch.nn.Linear(4, 4))
    raw = torch.nn.Module()
    block = torch.nn.Module()
    ff = _int8both_ff()
    block.ff = ff
    block.register_module("absent", None)
    raw.transformer_blocks = torch.nn.ModuleList([block])
    raw.eval()
    clone = int8_swiglu_fused.clone_fused_decoder(raw)
    assert raw.transformer_blocks[0].ff is ff
    assert clone.transformer_blocks[0] is not block
    assert clone.transformer_blocks[0].ff.w1.weight is ff.w1.weight
    assert clone.transformer_blocks[0].absent is None
    with pytest.raises(RuntimeError):   # grad mode is on: inference only
        clone.transformer_blocks[0].ff(torch.zeros(2, 4))
    raw.train()
    with pytest.raises(ValueError):
        int8_swiglu_fused.clone_fused_decoder(raw)


def test_norm_quant_clone_contracts(monkeypatch):
    """ref: tests/test_int8_norm_quant.py:29-59."""
    monkeypatch.setenv("MINIMAX_H3_VAE_DECODER_VIT_FP32_NORM", "0")
    with pytest.raises(ValueError):
        int8_norm_quant.clone_norm_quant_decoder(torch.nn.Module().eval())
    monkeypatch.setenv("MINIMAX_H3_VAE_DECODER_VIT_FP32_NORM", "1")
    with pytest.raises(ValueError):
        int8_norm_quant.clone_norm_quant_decoder(torch.nn.Module().eval(), 3)
    raw = torch.nn.Module()
    block = torch.nn.Module()
    block.use_scale = True
    block.norm1 = torch.nn.RMSNorm(2048).half()
    block.norm2 = torch.nn.RMSNorm(2048, eps=1e-5).half()
    block.attn = torch.nn.Identity()
    block.scale1 = torch.nn.Parameter(torch.ones(2048, dtype=torch.float16))
    block.scale2 = torch.nn.Parameter(torch.ones(2048, dtype=torch.float16))
    ff = _int8both_ff()
    block.ff = ff
    raw.transformer_blocks = torch.nn.ModuleList([block])
    raw.eval()
    result = int8_norm_quant.clone_norm_quant_decoder(raw)
    assert raw.transformer_blocks[0] is block
    assert isinstance(result.transformer_blocks[0], int8_norm_quant.NormQuantBlock)
    assert result.transformer_blocks[0].scale1 is block.scale1
    assert result.transformer_blocks[0].ff.w1.weight is ff.w1.weight
    assert result.transformer_blocks[0].fuse_ffn_up is False   # CPU parameters
    with pytest.raises(RuntimeError):
        result.transformer_blocks[0](torch.zeros(2, 2048))
    block.norm2 = torch.nn.RMSNorm(1024, eps=1e-5).half()
    with pytest.raises(ValueError):
        int8_norm_quant.NormQuantBlock(block)


def test_qkv_linear_validation_and_replacement_scope():
    """ref: tests/test_int8_qkv.py:16-49."""
    block = _attn_block()
    assert int8_qkv.qkv_linear(block)[1] is block.attn.original.to_qkv
    block.train()
    with pytest.raises(ValueError):
        int8_qkv.qkv_linear(block)
    with pytest.raises(ValueError):
        int8_qkv.qkv_linear(_attn_block(128))
    raw = torch.nn.Module()
    raw.transformer_blocks = torch.nn.ModuleList([_attn_block(), _attn_block()])
    raw.eval()
    clone = copy.deepcopy(raw)
    replacement = torch.nn.Identity()
    with patch.object(int8_qkv, "clone_norm_quant_decoder", return_value=clone), \
            patch.object(int8_qkv, "KitchenInt8Linear", return_value=replacement) as factory:
        result = int8_qkv.clone_qkv_int8_decoder(raw, indices=[1])
    assert isinstance(raw.transformer_blocks[1].attn.original.to_qkv, torch.nn.Linear)
    assert isinstance(result.transformer_blocks[0].attn.original.to_qkv, torch.nn.Linear)
    assert result.transformer_blocks[1].attn.original.to_qkv is replacement
    assert factory.call_count == 1 and factory.call_args.kwargs["require_cuda"]


def test_attention_out_validation_containers_and_scope():
    """ref: tests/test_int8_attention_out.py:18-60."""
    block = _attn_block()
    assert int8_attention_out.out_linear(block)[1] is block.attn.original.to_out
    block.train()
    with pytest.raises(ValueError):
        int8_attention_out.out_linear(block)
    with pytest.raises(ValueError):
        int8_attention_out.out_linear(_attn_block(128))
    block = _attn_block()
    block.attn.original.to_out = torch.nn.Identity()
    with pytest.raises(ValueError):
        int8_attention_out.out_linear(block)
    raw = _attn_block()
    raw.alias = raw.attn
    raw.register_buffer("probe", torch.ones(2))
    clone = clone_containers(raw)
    assert clone.attn is not raw.attn and clone.alias is clone.attn
    assert clone.probe is raw.probe
    assert clone.attn.original.to_out.weight is raw.attn.original.to_out.weight
    clone.probe = torch.zeros(2)
    assert torch.equal(raw.probe, torch.ones(2))
    raw = torch.nn.Module()
    raw.transformer_blocks = torch.nn.ModuleList([_attn_block(), _attn_block()])
    raw.eval()
    replacement = torch.nn.Identity()
    with patch.object(int8_attention_out, "KitchenInt8Linear", return_value=replacement) as factory:
        result = int8_attention_out.clone_attention_out_decoder(raw, indices=[1])
    for i in range(2):
        assert isinstance(raw.transformer_blocks[i].attn.original.to_out, torch.nn.Linear)
        assert (result.transformer_blocks[i].attn.original.to_qkv.weight
                is raw.transformer_blocks[i].attn.original.to_qkv.weight)
    assert isinstance(result.transformer_blocks[0].attn.original.to_out, torch.nn.Linear)
    assert result.transformer_blocks[1].attn.original.to_out is replacement
    assert factory.call_count == 1 and factory.call_args.kwargs["require_cuda"]


def test_kitchen_int8_ffn_modes_and_install():
    """ref: tests/test_kitchen_int8.py:105-127 (only the selected branch is replaced; inference only)
    and opt/kitchen_int8.py:283-310 (install validates every block before assigning)."""
    def gated():
        ff = torch.nn.Module()
        ff.use_gated, ff.act_fn = True, torch.nn.SiLU()
        ff.w1 = torch.nn.Linear(64, 128).half()
        ff.w2 = torch.nn.Linear(64, 64).half()
        return ff.eval()
    source = gated()
    cand = kitchen_int8.KitchenInt8FFN(source, "INT8w1").eval()
    assert isinstance(cand.w1, kitchen_int8.KitchenInt8Linear) and cand.w2 is source.w2
    assert cand.extra_weight_bytes == 128 * 64 + 128 * 4
    cand = kitchen_int8.KitchenInt8FFN(source, "INT8w2").eval()
    assert cand.w1 is source.w1 and isinstance(cand.w2, kitchen_int8.KitchenInt8Linear)
    with pytest.raises(ValueError):
        kitchen_int8.KitchenInt8FFN(source, "INT4")
    with pytest.raises(RuntimeError):
        kitchen_int8.KitchenInt8FFN(source).eval()(torch.zeros(2, 64, dtype=torch.float16))
    decoder = torch.nn.Module()
    blocks = [torch.nn.Module(), torch.nn.Module()]
    blocks[0].ff, blocks[1].ff = gated(), torch.nn.Linear(4, 4)   # the second block is not a gated FFN
    decoder.transformer_blocks = torch.nn.ModuleList(blocks)
    decoder.eval()
    original = decoder.transformer_blocks[0].ff
    with pytest.raises(ValueError):
        kitchen_int8.install_kitchen_int8_ffn(decoder, require_cuda=False)
    assert decoder.transformer_blocks[0].ff is original     # nothing assigned
    decoder.transformer_blocks[1].ff = gated()
    assert kitchen_int8.install_kitchen_int8_ffn(decoder, require_cuda=False) == 2
    assert all(isinstance(b.ff, kitchen_int8.KitchenInt8FFN) for b in decoder.transformer_blocks)


def _qk_attention(**overrides):
    attn = torch.nn.Module()
    attn.spatial_parallel = False
    attn.norm_q = torch.nn.RMSNorm(64, eps=1e-6, elementwise_affine=False)
    attn.norm_k = torch.nn.RMSNorm(64, eps=1e-6, elementwise_affine=False)
    attn.dim_head, attn.heads = 64, 2
    attn.to_qkv = torch.nn.Linear(128, 384)
    attn.to_out = torch.nn.Linear(128, 128)
    for k, v in overrides.items():
        setattr(attn, k, v)
    return attn.eval()


def test_qk_fusion_validation_delegation_and_clone(monkeypatch):
    """The fused-QK attention accepts only single-device, unaffined equal-eps RMSNorm QK norms with
    64-wide heads; without rotary tables it runs the original module; the clone leaves the caller's
    blocks untouched (ref: opt/decoder_fused_qk_rope.py:55-89)."""
    from h3vae_b200.opt.decoder_fused_qk_rope import FusedQKAttention, clone_with_qk_fusion
    for bad in (dict(spatial_parallel=True), dict(norm_q=torch.nn.LayerNorm(64)), dict(dim_head=128),
                dict(norm_k=torch.nn.RMSNorm(64, eps=1e-5, elementwise_affine=False)),
                dict(norm_q=torch.nn.RMSNorm(64, eps=1e-6))):
        with pytest.raises(ValueError):
            FusedQKAttention(_qk_attention(**bad))
    calls = []

    class Recording(torch.nn.Module):
        def forward(self, x, rotary, pack_info):
            calls.append((rotary, pack_info))
            return x

    attn = _qk_attention()
    attn.forward = Recording().forward
    fused = FusedQKAttention(attn)
    x = torch.zeros(1, 3, 128)
    assert fused(x) is x and calls == [(None, {})]
    raw = torch.nn.Module()
    block = torch.nn.Module()
    block.attn = _qk_attention()
    raw.transformer_blocks = torch.nn.ModuleList([block])
    raw.eval()
    result = clone_with_qk_fusion(raw)
    assert raw.transformer_blocks[0] is block and isinstance(block.attn, torch.nn.Module)
    assert not isinstance(block.attn, FusedQKAttention)
    assert isinstance(result.transformer_blocks[0].attn, FusedQKAttention)
    assert result.transformer_blocks[0].attn.original is block.attn
    monkeypatch.setenv("MINIMAX_H3_VAE_DECODER_VIT_FP32_NORM", "0")
    with pytest.raises(ValueError):
        clone_with_qk_fusion(raw)


def test_final_norm_adapter_shares_parameters_and_keeps_tensor_path():
    """ref: tests/test_int8_norm1_quant.py:33-64."""
    from h3vae_b200.opt import int8_norm1_quant as norm1
    source = torch.nn.LayerNorm(2048, eps=1e-5, dtype=torch.float16).eval()
    adapter = norm1._FinalNormAdapter(source).eval()
    assert set(adapter.state_dict()) == set(source.state_dict())
    assert adapter.weight is source.weight and adapter.bias is source.bias
    with torch.inference_mode():
        x = torch.randn(2, 7, 2048, dtype=torch.float16)
        assert torch.equal(adapter(x), source(x))
        adapter.to(dtype=torch.float32)
        assert adapter.weight is source.weight
        assert torch.equal(adapter(x.float()), source(x.float()))
    adapter = norm1._FinalNormAdapter(torch.nn.LayerNorm(2048, eps=1e-5, dtype=torch.float16).eval()).eval()
    old = torch.__future__.get_overwrite_module_params_on_conversion()
    try:
        torch.__future__.set_overwrite_module_params_on_conversion(True)
        adapter.to(dtype=torch.float32)
    finally:
        torch.__future__.set_overwrite_module_params_on_conversion(old)
    with torch.inference_mode():
        y = adapter(torch.randn(2, 7, 2048))
    assert y.dtype == torch.float32 and bool(torch.isfinite(y).all())


def test_carry_safe_unpad():
    """ref: tests/test_int8_norm1_quant.py:77-93."""
    from unittest.mock import Mock

    from h3vae_b200.opt import int8_norm1_quant as norm1
    original = Mock(side_effect=lambda states, pad: states)
    unpad = norm1._carry_safe_unpad(original)
    carry = (object(), object(), object())
    assert unpad(carry, 0) is carry
    original.reset_mock()
    with pytest.raises(RuntimeError, match="zero sequence padding"):
        unpad(carry, 1)
    original.assert_not_called()
    tensor = torch.empty(2, 5, 3)
    assert unpad(tensor, 1) is tensor
    original.assert_called_once_with(tensor, 1)
    with pytest.raises(RuntimeError, match="preserve final residual carry"):
        norm1._carry_safe_unpad(lambda s, p: tuple(list(s)))((object(), object(), object()), 0)


def test_norm1_device_gate_and_clone_guards():
    """The chain runs on sm_100 only (ref: tests/test_int8_norm1_quant.py:95-103, with this build's
    gate); the clone refuses training decoders and wrong block counts and, disabled, returns a plain
    container clone (ref: opt/int8_norm1_quant.py:282-296)."""
    from h3vae_b200.opt import int8_norm1_quant as norm1
    assert norm1.supports_norm1_quant("cpu") is False
    for capability, expected in (((10, 0), True), ((12, 0), False), ((9, 0), False)):
        norm1._device_supports_norm1_quant.cache_clear()
        with patch.object(torch.cuda, "is_available", return_value=True), \
                patch.object(torch.cuda, "get_device_capability", return_value=capability):
            assert norm1.supports_norm1_quant("cuda:0") is expected
    norm1._device_supports_norm1_quant.cache_clear()
    raw = torch.nn.Module()
    raw.transformer_blocks = torch.nn.ModuleList([torch.nn.Linear(2, 2) for _ in range(36)])
    raw.train()
    with pytest.raises(ValueError):
        norm1.clone_norm1_quant_decoder(raw)
    raw.eval()
    result = norm1.clone_norm1_quant_decoder(raw)
    assert result._h3vae_norm1_quant_enabled is False
    assert result is not raw and result.transformer_blocks[0] is not raw.transformer_blocks[0]
    assert result.transformer_blocks[0].weight is raw.transformer_blocks[0].weight
    with pytest.raises(RuntimeError):   # enabling needs an sm_100 device
        norm1.clone_norm1_quant_decoder(raw, enabled=True)
    raw.transformer_blocks = torch.nn.ModuleList([torch.nn.Linear(2, 2) for _ in range(35)])
    with pytest.raises(ValueError):
        norm1.clone_norm1_quant_decoder(raw)


def _fake_encoder():
    torch.manual_seed(0)
    enc = torch.nn.Module()
    enc.gradient_checkpointing, enc.use_fused_norm = False, False
    enc.conv_in = torch.nn.Conv3d(3, 8, 1)
    stages = []
    for down in (True, True, False):
        stage = torch.nn.Module()
        stage.block = torch.nn.ModuleList([torch.nn.Conv3d(8, 8, (1, 3, 3), padding=(0, 1, 1))])
        if down:
            stage.downsample = torch.nn.Conv3d(8, 8, (1, 2, 2), stride=(1, 2, 2))
        stages.append(stage)
    enc.down = torch.nn.ModuleList(stages)
    enc.norm_out = torch.nn.GroupNorm(2, 8)
    enc.conv_out = torch.nn.Conv3d(8, 4, 1)
    return enc.eval(), torch.nn.Conv3d(4, 4, 1).eval()


@pytest.mark.parametrize("cut,batch,token_drop", [(1, 1, 0), (2, 2, 0), (2, 4, 3), (1, 2, 1)])
def test_encode_staged_equals_per_clip_encoding(cut, batch, token_drop):
    """Staged clip batching (ref: opt/encoder_staged_batch.py:39-57) equals encoding each padded
    17-frame clip on its own and concatenating in time, then dropping token_drop latent frames."""
    from h3vae_b200.opt.encoder_staged_batch import EncoderPrefix, EncoderSuffix, encode_staged
    enc, quant = _fake_encoder()
    prefix, suffix = EncoderPrefix(enc, cut), EncoderSuffix(enc, quant, cut)
    video = torch.randn(1, 3, 40, 16, 16, generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        got = encode_staged(video, prefix, suffix, clip_length=17, token_drop=token_drop, batch_size=batch, cut=cut)
        padded = torch.cat([video, video[:, :, -1:].repeat(1, 1, 11, 1, 1)], dim=2)
        ref = torch.cat([suffix(prefix(padded[:, :, t:t + 17])) for t in (0, 17, 34)], dim=2)
    ref = ref[:, :, :-token_drop] if token_drop else ref
    assert got.shape == ref.shape
    assert torch.allclose(got, ref, atol=1e-5, rtol=1e-5)


def test_encode_staged_guards():
    from h3vae_b200.opt.encoder_staged_batch import EncoderPrefix, EncoderSuffix, encode_staged
    enc, quant = _fake_encoder()
    prefix, suffix = EncoderPrefix(enc, 2), EncoderSuffix(enc, quant, 2)
    with pytest.raises(ValueError):
        EncoderPrefix(enc, 3)
    enc.use_fused_norm = True
    with pytest.raises(ValueError):
        EncoderPrefix(enc, 1)
    with pytest.raises(ValueError):   # batch-one videos only
        encode_staged(torch.zeros(2, 3, 17, 8, 8), prefix, suffix, clip_length=17, token_drop=0, batch_size=1, cut=2)
    with pytest.raises(ValueError):   # unvalidated (cut, batch) pair
        encode_staged(torch.zeros(1, 3, 17, 8, 8), prefix, suffix, clip_length=17, token_drop=0, batch_size=4, cut=1)
