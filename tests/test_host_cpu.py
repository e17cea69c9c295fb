"""Host-side checks that need no GPU: the C-ABI library exports, the option validation policy of
the runtime, the ComfyUI node surface, and the argument checks of the reference-facing op mirrors.
"""
from __future__ import annotations

import re
import sys

import numpy as np
import pytest
import torch

from conftest import ROOT


def _header_symbols():
    text = (ROOT / "include" / "h3vae_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    return sorted(set(re.findall(r"\b(h3b_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    from h3vae_b200 import _lib, build_lib
    build_lib.build()
    lib = _lib.load()
    symbols = _header_symbols()
    assert len(symbols) == 38
    missing = [s for s in symbols if not hasattr(lib, s)]
    assert not missing, f"declared in the header but not exported: {missing}"
    assert set(symbols) == set(_lib._SIGNATURES), "ctypes signature table out of sync with the header"
    assert lib.h3b_abi_version() == 100


def test_workspace_sizes_scale_with_shape():
    from h3vae_b200 import _lib
    lib = _lib.load()
    small = lib.h3b_norm_workspace_size(1, 128, 19, 64, 64)
    big = lib.h3b_norm_workspace_size(4, 128, 19, 258, 258)
    assert 0 < small < big
    assert lib.h3b_quantize_tensor_workspace_size() > 0


def test_product_modules_do_not_import_the_oracle():
    pkg = ROOT / "comfyui-h3vae-pyopt_b200"
    for path in list(pkg.rglob("*.py")) + list(pkg.rglob("*.cu")) + list(pkg.rglob("*.cuh")):
        assert "oracle" not in path.read_text().replace("oracle-free", ""), f"{path} references the oracle"


# ---------------------------------------------------------------------------
# Option validation (ref: h3vae_runtime.py:50-181): fail before any weight is built, no fallback
# ---------------------------------------------------------------------------
GOOD = dict(cuda_available=True, capability=(10, 0), hip=None)


def test_int8_decode_validation_policy():
    from h3vae_b200.runtime import _validate_int8_decode_options as v
    v(enabled=False, fast_linear=True, device="cpu", dtype=torch.float32)       # disabled: nothing checked
    v(enabled=True, fast_linear=False, device="cuda", dtype=torch.float16, library_available=True, **GOOD)
    with pytest.raises(ValueError, match="mutually exclusive"):
        v(enabled=True, fast_linear=True, device="cuda", dtype=torch.float16, **GOOD)
    with pytest.raises(RuntimeError, match="CUDA device"):
        v(enabled=True, fast_linear=False, device="cpu", dtype=torch.float16, **GOOD)
    with pytest.raises(RuntimeError, match="fp16"):
        v(enabled=True, fast_linear=False, device="cuda", dtype=torch.float32, **GOOD)
    with pytest.raises(RuntimeError, match="ROCm"):
        v(enabled=True, fast_linear=False, device="cuda", dtype=torch.float16,
          **{**GOOD, "hip": "6.2"})
    with pytest.raises(RuntimeError, match="available CUDA GPU"):
        v(enabled=True, fast_linear=False, device="cuda", dtype=torch.float16,
          **{**GOOD, "cuda_available": False})
    with pytest.raises(RuntimeError, match="sm_100"):
        v(enabled=True, fast_linear=False, device="cuda", dtype=torch.float16,
          **{**GOOD, "capability": (12, 0)})
    with pytest.raises(RuntimeError, match="no fallback"):
        v(enabled=True, fast_linear=False, device="cuda", dtype=torch.float16, library_available=False, **GOOD)


def test_int8_encode_and_fusion_validation_policy():
    from h3vae_b200.runtime import _validate_decode_fusions_options, _validate_int8_encode_options
    _validate_int8_encode_options(enabled=True, device="cuda", dtype=torch.float16, library_available=True, **GOOD)
    with pytest.raises(RuntimeError, match="int8_encode requires dtype=fp16"):
        _validate_int8_encode_options(enabled=True, device="cuda", dtype=torch.float32, **GOOD)
    with pytest.raises(RuntimeError, match="int8_encode requires a CUDA device"):
        _validate_int8_encode_options(enabled=True, device="cpu", dtype=torch.float16, **GOOD)
    with pytest.raises(RuntimeError, match="sm_100"):
        _validate_int8_encode_options(enabled=True, device="cuda", dtype=torch.float16,
                                      **{**GOOD, "capability": (9, 0)})
    with pytest.raises(ValueError, match="mutually exclusive"):
        _validate_decode_fusions_options(enabled=True, device="cuda", dtype=torch.float16, fast_linear=True)
    with pytest.raises(RuntimeError, match="fp16"):
        _validate_decode_fusions_options(enabled=True, device="cuda", dtype=torch.float32, fast_linear=False)
    _validate_decode_fusions_options(enabled=True, device="cuda", dtype=torch.float16, fast_linear=False, **GOOD)


@pytest.mark.parametrize("kwargs, exc, match", [
    (dict(fast_linear=True), ValueError, "fast_linear"),
    (dict(encoder_tile_size=24), ValueError, "multiple of 16"),
    (dict(encoder_tile_size=32), ValueError, "exceed"),
    (dict(encoder_staged_batch=3), ValueError, "1, 2 or 4"),
    (dict(tile_batch=-1), ValueError, "non-negative"),
    (dict(model_code_dir="/nonexistent"), NotImplementedError, "synthetic"),
    (dict(dtype=torch.bfloat16), RuntimeError, "fp16 or fp32"),
    (dict(dtype=torch.float32, decode_fusions=True, device="cpu"), RuntimeError, "fp16"),
    (dict(int8_decode=True, device="cpu"), RuntimeError, "CUDA device"),
    (dict(act_scale_mode="channel"), ValueError, "act_scale_mode"),
])
def test_runtime_rejects_bad_options_before_building(kwargs, exc, match):
    from h3vae_b200.runtime import H3VAEPyOptRuntime
    with pytest.raises(exc, match=match):
        H3VAEPyOptRuntime(**{"device": "cpu", **kwargs})


# ---------------------------------------------------------------------------
# ComfyUI node surface (ref: h3vae_nodes.py:35-197)
# ---------------------------------------------------------------------------
def test_node_inputs_and_mappings():
    import importlib.util
    spec = importlib.util.spec_from_file_location("h3b_custom_nodes", ROOT / "comfyui-h3vae-pyopt_b200" / "__init__.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    node = mod.NODE_CLASS_MAPPINGS["H3VAEPyOptLoader"]
    assert "H3VAEPyOptLoader" in mod.NODE_DISPLAY_NAME_MAPPINGS
    types = node.INPUT_TYPES()
    required = {k: v[1].get("default") for k, v in types["required"].items()}
    assert required == {"vae_name": "use default", "dtype": "fp16", "decoder_tile_size": 256, "tile_batch": 2,
                        "compile_decoder": True, "compile_encoder": True, "encoder_staged_batch": 4,
                        "cudnn_benchmark": True, "warmup": "none", "warmup_frames": 124, "warmup_width": 1344,
                        "warmup_height": 768, "log_calls": True}
    optional = {k: v[1].get("default") for k, v in types["optional"].items()}
    assert optional.keys() == {"encoder_tile_size", "fast_linear", "decode_fusions", "int8_decode", "int8_encode",
                               "model_code_dir", "weights_path", "act_scale_mode"}
    assert optional["act_scale_mode"] == "tensor"
    assert node.RETURN_TYPES == ("VAE",) and node.FUNCTION == "load"
    with pytest.raises(ValueError, match="mutually exclusive"):
        node().load("use default", "fp16", 256, 2, True, True, 4, True, "none", 124, 1344, 768, True,
                    fast_linear=True, int8_decode=True)


# ---------------------------------------------------------------------------
# opt/* mirrors: argument checks that run before any kernel, and static weight quantization
# ---------------------------------------------------------------------------
def test_opt_mirror_argument_checks():
    from h3vae_b200.opt import fp16_finalize, int8_ffn_up_fused, int8_swiglu_fused
    with pytest.raises(ValueError, match="even width"):
        int8_swiglu_fused.validate_input(torch.zeros(4, 7, dtype=torch.float16))
    with pytest.raises(ValueError, match="FP16"):
        int8_swiglu_fused.validate_input(torch.zeros(4, 8))
    q = torch.zeros(4, 64, dtype=torch.int8)
    with pytest.raises(ValueError, match="dimensions"):
        int8_swiglu_fused.prequantized_linear(q, torch.ones(4, 1), torch.zeros(8, 32, dtype=torch.int8), torch.ones(8))
    with pytest.raises(ValueError, match="one scale"):
        int8_swiglu_fused.prequantized_linear(q, torch.ones(3, 1), torch.zeros(8, 64, dtype=torch.int8), torch.ones(8))
    with pytest.raises(ValueError, match=r"\[2F, K\]"):
        int8_ffn_up_fused.validate_prequantized(q, torch.ones(4, 1), torch.zeros(7, 64, dtype=torch.int8),
                                                torch.ones(7), None)
    x = torch.zeros(1, 3, 2, 4, 4)
    with pytest.raises(ValueError, match="channel constants"):
        fp16_finalize.validate(x, torch.ones(3, dtype=torch.float16), torch.zeros(3))
    with pytest.raises(ValueError, match="B,3,T,H,W"):
        fp16_finalize.validate(torch.zeros(1, 4, 2, 4, 4), torch.ones(3), torch.zeros(3))


def test_kitchen_static_weight_matches_oracle():
    from oracle import h3vae_oracle as O
    from h3vae_b200.opt.kitchen_int8 import KitchenInt8Linear
    lin = torch.nn.Linear(256, 96).half()
    with torch.no_grad():
        lin.weight[5].zero_()
    mod = KitchenInt8Linear(lin).eval()
    q_ref, s_ref = O.quantize_rowwise_weight(lin.weight.detach())
    np.testing.assert_array_equal(mod.qweight.numpy(), q_ref.numpy())
    np.testing.assert_array_equal(mod.weight_scale.numpy(), s_ref.reshape(-1).numpy())
    assert mod.weight_scale[5] == 1.0 and not mod.qweight[5].any()
    with pytest.raises(RuntimeError, match="no_grad"):
        mod(torch.zeros(2, 256, dtype=torch.float16))
    with torch.no_grad(), pytest.raises(ValueError, match="K=128"):
        mod(torch.zeros(2, 128, dtype=torch.float16))
    lin.weight.data[0, 0] = float("inf")
    with pytest.raises(ValueError, match="non-finite"):
        KitchenInt8Linear(lin)


def test_oracle_per_token_quantization_known_answer():
    """One scale per position: absmax over the channels * fp32(1/127); half-away rounding."""
    from oracle import h3vae_oracle as O
    x = np.zeros((1, 3, 1, 1, 2), np.float16)
    x[0, :, 0, 0, 0] = [1.0, -2.0, 0.5]        # position 0: absmax 2
    x[0, :, 0, 0, 1] = [0.0, 0.0, 0.0]         # position 1: all zero -> scale 1
    q, s = O.quantize_activation_per_token(x)
    s0 = np.float32(2.0) * np.float32(1.0 / 127.0)
    assert s[0, 0, 0, 0] == s0 and s[0, 0, 0, 1] == 1.0
    expect = np.where(x[0, :, 0, 0, 0] / s0 >= 0, np.floor(x[0, :, 0, 0, 0] / s0 + 0.5),
                      -np.floor(-x[0, :, 0, 0, 0] / s0 + 0.5))
    assert np.array_equal(q[0, :, 0, 0, 0], expect.astype(np.int8)) and q[0, 1, 0, 0, 0] == -127
    assert not q[..., 1].any()
    # per-token conv of a constant-scale input equals the per-tensor conv
    rng = np.random.default_rng(1)
    qa = rng.integers(-127, 128, (1, 4, 3, 4, 4), dtype=np.int8)
    sc = np.full((1, 3, 4, 4), 0.02, np.float32)
    qw = rng.integers(-127, 128, (2, 27 * 4), dtype=np.int8)
    ws = np.array([0.001, 0.002], np.float32)
    a = O.conv3d_per_token(qa, sc, qw, ws, (3, 3, 3)).astype(np.float32)
    b = O.conv_epilogue(O.conv3d_int_acc(qa, qw, (3, 3, 3)), np.float32(0.02), ws, None).astype(np.float32)
    assert np.allclose(a, b, atol=2e-3, rtol=2e-3)


def _gated_decoder():
    ff = torch.nn.Module()
    ff.use_gated, ff.act_fn = True, torch.nn.SiLU()
    ff.w1 = torch.nn.Linear(4, 16, dtype=torch.float16)
    ff.w2 = torch.nn.Linear(8, 4, dtype=torch.float16)
    block = torch.nn.Module()
    block.ff, block.attn = ff, torch.nn.Identity()
    raw = torch.nn.Module()
    raw.transformer_blocks = torch.nn.ModuleList([block])
    return raw.eval()


def test_fp16_swiglu_mirror_module_swap():
    """ref: tests/test_fp16_swiglu_gemm.py:15-27 (clone keeps the original and shares the weights;
    training mode and non-SiLU FFNs are refused)."""
    from h3vae_b200.opt.fp16_swiglu_gemm import FusedFP16FFN, clone_fp16_decoder
    raw = _gated_decoder()
    cand = clone_fp16_decoder(raw, (128, 64, 64, 4, 2))
    assert not isinstance(raw.transformer_blocks[0].ff, FusedFP16FFN)
    assert isinstance(cand.transformer_blocks[0].ff, FusedFP16FFN)
    assert cand.transformer_blocks[0].ff.w1 is not raw.transformer_blocks[0].ff.w1
    assert cand.transformer_blocks[0].ff.w1.weight is raw.transformer_blocks[0].ff.w1.weight
    assert set(cand.state_dict()) == set(raw.state_dict())
    raw.train()
    with pytest.raises(ValueError):
        clone_fp16_decoder(raw, (128, 64, 64, 4, 2))
    raw.eval()
    raw.transformer_blocks[0].ff.act_fn = torch.nn.GELU()
    with pytest.raises(ValueError):
        clone_fp16_decoder(raw, (128, 64, 64, 4, 2))


def test_fp16_swiglu_mirror_guards():
    """ref: tests/test_fp16_swiglu_gemm.py:29-42 (CPU tensors and every shape / dtype / config
    violation raise ValueError before any launch)."""
    from h3vae_b200.opt.fp16_swiglu_gemm import fused_w1_swiglu, validate
    x = torch.ones(2, 4, dtype=torch.float16)
    w = torch.ones(8, 4, dtype=x.dtype)
    validate(x, w, None, (64, 64, 64, 4, 3))
    with pytest.raises(ValueError, match="CUDA"):
        fused_w1_swiglu(x, w)
    for a, b, bias, c in [(x.float(), w, None, (64, 64, 64, 4, 3)), (x, w[:7], None, (64, 64, 64, 4, 3)),
                          (x, w, torch.zeros(7, dtype=x.dtype), (64, 64, 64, 4, 3)),
                          (x, w, None, (64, 64, 64, 1, 3)), (x, w, None, (64, 64, 64, 4)),
                          (x[:0], w, None, (64, 64, 64, 4, 3))]:
        with pytest.raises(ValueError):
            validate(a, b, bias, c)


def test_oracle_fp16_block_chain_against_independent_fp32_torch():
    """Pins the oracle composition that the fp16 block-chain GPU test compares against: the same
    two blocks written independently in fp32 PyTorch (no fp16 rounding points) agree within 1e-3
    relative L2."""
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from test_model_gpu import _oracle_fp16_chain

    from h3vae_b200.model import DecoderConfig, H3Decoder
    cfg = DecoderConfig(hidden=256, heads=4, blocks=2, ffn=512, up_channels=(128,), up_spatial=(True,),
                        up_temporal=(True,))
    dec = H3Decoder(cfg, device="cpu", seed=3, int8=False)
    grid = (2, 8, 16)
    x = torch.randn(2, 256, 256, generator=torch.Generator().manual_seed(9)).half()
    ref = torch.from_numpy(_oracle_fp16_chain(dec, x, grid))
    b, n, d = x.shape
    cos, sin = (t.float() for t in dec._rope(b, *grid))
    r = cos.shape[-1]
    xs = x.float().reshape(b * n, d)

    def rms(t, w):
        return t * torch.rsqrt((t * t).mean(-1, keepdim=True) + cfg.eps) * w.float()

    def norm_rope(v):
        v = v * torch.rsqrt((v * v).mean(-1, keepdim=True) + cfg.qk_eps)
        rot = torch.cat([-v[..., r // 2:r], v[..., : r // 2]], -1)
        return torch.cat([v[..., :r] * cos + rot * sin, v[..., r:]], -1)

    for blk in dec.blocks:
        qkv = (rms(xs, blk.norm1_w) @ blk.qkv_w.float().T + blk.qkv_b.float()).view(b, n, cfg.heads, 3, 64)
        q, k, v = norm_rope(qkv[:, :, :, 0]), norm_rope(qkv[:, :, :, 1]), qkv[:, :, :, 2]
        p = torch.softmax(q.transpose(1, 2) @ k.transpose(1, 2).transpose(-1, -2) / 8, -1)
        att = (p @ v.transpose(1, 2)).transpose(1, 2).reshape(b * n, d)
        h = xs + (att @ blk.out_w.float().T + blk.out_b.float()) * blk.scale1.float()
        ff = rms(h, blk.norm2_w) @ blk.up_w.float().T + blk.up_b.float()
        g, u = ff[:, : cfg.ffn], ff[:, cfg.ffn:]
        xs = h + ((g * torch.sigmoid(g) * u) @ blk.down_w.float().T + blk.down_b.float()) * blk.scale2.float()
    y = torch.nn.functional.layer_norm(xs, (d,), dec.ln_w.float(), dec.ln_b.float(), cfg.eps).view(b, n, d)
    assert ((y.double() - ref).norm() / ref.norm()).item() < 1e-3


def test_build_comfy_vae_with_a_stand_in_comfy(monkeypatch):
    """The comfy.sd.VAE wrapper (ref: h3vae_runtime.py:720-806) against stand-in comfy modules: the
    latent / pixel ratios follow the runtime's clip geometry, input pixels map [0,1] -> [-1,1], the
    runtime is the patched first-stage model, and a non-FP16 VAE dtype is refused."""
    import types

    from h3vae_b200.model import DecoderConfig, EncoderConfig
    from h3vae_b200.runtime import H3VAEPyOptRuntime, build_comfy_vae

    mm = types.ModuleType("comfy.model_management")
    mm.vae_device = lambda: torch.device("cpu")
    mm.vae_offload_device = lambda: torch.device("cpu")
    mm.vae_dtype = lambda device, dtypes: dtypes[0]
    mm.intermediate_device = lambda: torch.device("cpu")
    mm.dtype_size = lambda dtype: 2
    mp = types.ModuleType("comfy.model_patcher")

    class CoreModelPatcher:
        def __init__(self, model, load_device, offload_device):
            self.model, self.load_device, self.offload_device = model, load_device, offload_device

    mp.CoreModelPatcher = CoreModelPatcher
    sd = types.ModuleType("comfy.sd")

    class VAE:
        def model_size(self):
            self.size = 1234
            return self.size

    sd.VAE = VAE
    comfy = types.ModuleType("comfy")
    comfy.model_management, comfy.model_patcher, comfy.sd = mm, mp, sd
    for name, module in (("comfy", comfy), ("comfy.model_management", mm), ("comfy.model_patcher", mp),
                         ("comfy.sd", sd)):
        monkeypatch.setitem(sys.modules, name, module)

    runtime = H3VAEPyOptRuntime(device="cpu", log_calls=False, compile_decoder=False, compile_encoder=False,
                                encoder_config=EncoderConfig(channels=(32, 32, 32, 32), blocks_per_stage=1,
                                                             int8_stages=()),
                                decoder_config=DecoderConfig(hidden=64, heads=1, blocks=1, ffn=128,
                                                             up_channels=(32, 32, 32)))
    vae = build_comfy_vae(runtime)
    tpc, ratio = runtime.tokens_per_clip, runtime.decoder.spatial_ratio
    assert isinstance(vae, VAE) and vae.patcher.model is runtime and vae.size == 1234
    assert vae.latent_channels == runtime.latent_channels and vae.handles_tiling
    # the reference's temporal contract: frames 17k+5 <-> latents 5k+2, one frame <-> one latent
    # (ref: h3vae_runtime.py:739-742)
    assert tpc == 5 and vae.upscale_ratio[1:] == (ratio, ratio) and vae.downscale_ratio[1:] == (ratio, ratio)
    assert vae.upscale_ratio[0](37) == 124 and vae.downscale_ratio[0](124) == 37
    assert vae.upscale_ratio[0](2) == 5 and vae.downscale_ratio[0](5) == 2
    assert vae.upscale_ratio[0](1) == 1 and vae.downscale_ratio[0](1) == 1
    for k in range(6):
        assert vae.upscale_ratio[0](5 * k + 2) == 17 * k + 5 and vae.downscale_ratio[0](17 * k + 5) == 5 * k + 2
    assert vae.upscale_index_formula == (4, ratio, ratio) and vae.downscale_index_formula == (4, ratio, ratio)
    assert vae.working_dtypes == [torch.float16, torch.float32]
    x = torch.rand(1, 3, 2, 4, 4)
    assert torch.equal(vae.process_input(x), x * 2.0 - 1.0) and vae.process_output(x) is x
    assert vae.memory_used_decode((1, 16, tpc, 8, 8), torch.float16) > vae.memory_used_decode((1, 16, tpc, 4, 4),
                                                                                            torch.float16)
    mm.vae_dtype = lambda device, dtypes: torch.float32
    assert build_comfy_vae(runtime).vae_dtype == torch.float32   # fp32 is allowed outside the INT8 modes
    mm.vae_dtype = lambda device, dtypes: torch.bfloat16
    with pytest.raises(RuntimeError, match="FP16"):
        build_comfy_vae(runtime)
