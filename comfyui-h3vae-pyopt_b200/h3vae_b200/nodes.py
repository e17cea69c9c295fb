"""ComfyUI node: the H3 video VAE loader backed by the B200 runtime.

Same node class, inputs, defaults, cache key and warmup policy as the reference's
`H3VAEPyOptLoader` (h3vae_nodes.py:35-191), so an existing workflow keeps its widget values.
Options that select the reference's compile/Triton stack (compile_decoder, compile_encoder,
cudnn_benchmark) are accepted and have no effect on the precompiled sm_100a kernels;
fast_linear (a comfy-kitchen FP16 path) is refused by the runtime.
"""
from __future__ import annotations

import logging

import torch

from .runtime import DEFAULT_MODEL_CODE_DIR, DEFAULT_WEIGHTS_FALLBACK, H3VAEPyOptRuntime, build_comfy_vae

logger = logging.getLogger("ComfyUI_H3VAE_B200")

# Built VAEs keyed by every load option, so re-queueing a workflow reuses the loaded runtime.
_VAE_CACHE: dict[tuple, object] = {}


def _folder_paths():
    import folder_paths  # ComfyUI module, only present inside ComfyUI
    return folder_paths


def _resolve_weights(vae_name: str, weights_path: str) -> str:
    """ref: h3vae_nodes.py:25-32."""
    if weights_path:
        return weights_path
    if vae_name == "use default":
        # An empty path selects the runtime's H3-structured synthetic weights.
        return DEFAULT_WEIGHTS_FALLBACK
    return _folder_paths().get_full_path_or_raise("vae", vae_name)


class H3VAEPyOptLoader:
    """Load the H3 video VAE on the B200 INT8 runtime."""

    @classmethod
    def INPUT_TYPES(cls):
        try:
            vae_files = _folder_paths().get_filename_list("vae")
        except Exception:  # noqa: BLE001 - outside ComfyUI there is no model folder
            vae_files = []
        choices = ["use default"] + list(vae_files)
        return {
            "required": {
                "vae_name": (choices, {"default": "use default"}),
                "dtype": (["fp16", "fp32"], {"default": "fp16"}),
                "decoder_tile_size": ("INT", {"default": 256, "min": 128, "max": 1024, "step": 16}),
                "tile_batch": ("INT", {"default": 2, "min": 0, "max": 8, "step": 1}),
                "compile_decoder": ("BOOLEAN", {"default": True}),
                "compile_encoder": ("BOOLEAN", {"default": True}),
                "encoder_staged_batch": ([1, 2, 4], {"default": 4}),
                "cudnn_benchmark": ("BOOLEAN", {"default": True}),
                "warmup": (["none", "decode", "encode", "both"], {"default": "none"}),
                "warmup_frames": ("INT", {"default": 124, "min": 1, "max": 1000}),
                "warmup_width": ("INT", {"default": 1344, "min": 64, "max": 4096, "step": 16}),
                "warmup_height": ("INT", {"default": 768, "min": 64, "max": 4096, "step": 16}),
                "log_calls": ("BOOLEAN", {"default": True}),
            },
            "optional": {
                "encoder_tile_size": ("INT", {"default": 0, "min": 0, "max": 1024, "step": 16,
                                              "tooltip": "0 = auto: 672 up to 672x672, else 256."}),
                "fast_linear": ("BOOLEAN", {"default": False}),
                "decode_fusions": ("BOOLEAN", {"default": False}),
                "int8_decode": ("BOOLEAN", {"default": False,
                                            "tooltip": "tcgen05 INT8 decoder transformer (QKV+RoPE, attention, "
                                                       "SwiGLU FFN) on sm_100a."}),
                "int8_encode": ("BOOLEAN", {"default": False,
                                            "tooltip": "tcgen05 INT8 causal conv3d encoder on sm_100a."}),
                "act_scale_mode": (["tensor", "token"], {"default": "tensor",
                                                          "tooltip": "INT8 encoder activation scales: one per tensor "
                                                                     "(the reference's scheme) or one per "
                                                                     "spatio-temporal position."}),
                "model_code_dir": ("STRING", {"default": DEFAULT_MODEL_CODE_DIR}),
                "weights_path": ("STRING", {"default": ""}),
            },
        }

    RETURN_TYPES = ("VAE",)
    FUNCTION = "load"
    CATEGORY = "MiniMax_H3/Acceleration"
    DESCRIPTION = ("Load the H3 video VAE on B200-native sm_100a kernels: INT8 tcgen05 conv3d encoder, "
                   "INT8 tcgen05 decoder transformer, fused norm/quant producers.")

    def load(self, vae_name, dtype, decoder_tile_size, tile_batch, compile_decoder, compile_encoder,
             encoder_staged_batch, cudnn_benchmark, warmup, warmup_frames, warmup_width, warmup_height,
             log_calls, model_code_dir=DEFAULT_MODEL_CODE_DIR, weights_path="", encoder_tile_size=0,
             fast_linear=False, int8_decode=False, int8_encode=False, decode_fusions=False, act_scale_mode="tensor"):
        """ref: h3vae_nodes.py:134-191."""
        if bool(fast_linear) and bool(int8_decode):
            raise ValueError("int8_decode and fast_linear are mutually exclusive; choose one")
        key = (vae_name, weights_path, dtype, int(decoder_tile_size), int(encoder_tile_size), int(tile_batch),
               bool(compile_decoder), bool(compile_encoder), int(encoder_staged_batch), model_code_dir,
               bool(log_calls), bool(fast_linear), bool(int8_decode), bool(int8_encode), bool(decode_fusions),
               act_scale_mode)
        vae = _VAE_CACHE.get(key)
        if vae is None:
            weights = _resolve_weights(vae_name, weights_path)
            torch.backends.cudnn.benchmark = bool(cudnn_benchmark)
            runtime = H3VAEPyOptRuntime(
                model_code_dir=model_code_dir, weights_path=weights, device="cuda",
                dtype=torch.float16 if dtype == "fp16" else torch.float32,
                decoder_tile_size=int(decoder_tile_size), encoder_tile_size=int(encoder_tile_size),
                tile_batch=int(tile_batch), compile_decoder=bool(compile_decoder),
                compile_encoder=bool(compile_encoder), encoder_staged_batch=int(encoder_staged_batch),
                fast_linear=bool(fast_linear), int8_decode=bool(int8_decode), int8_encode=bool(int8_encode),
                decode_fusions=bool(decode_fusions), log_calls=bool(log_calls), act_scale_mode=act_scale_mode)
            vae = build_comfy_vae(runtime)
            _VAE_CACHE[key] = vae
            logger.info("[H3VAE-B200] loaded %s (%s, tile=%d, batch=%d)", weights or "synthetic weights", dtype,
                        decoder_tile_size, tile_batch)
        runtime = vae.first_stage_model
        if warmup != "none" and not getattr(runtime, "_warmed_up", False):
            try:
                runtime.warmup(int(warmup_frames), int(warmup_width), int(warmup_height), mode=warmup)
                runtime._warmed_up = True
            except Exception as exc:  # noqa: BLE001 - best effort unless an explicit INT8 mode was asked for
                if runtime.int8_decode or runtime.int8_encode or runtime.decode_fusions:
                    raise RuntimeError("explicit optimized VAE warmup failed; no fallback was applied") from exc
                logger.warning("[H3VAE-B200] warmup failed (%s: %s)", type(exc).__name__, exc)
        return (vae,)


NODE_CLASS_MAPPINGS = {"H3VAEPyOptLoader": H3VAEPyOptLoader}
NODE_DISPLAY_NAME_MAPPINGS = {"H3VAEPyOptLoader": "MiniMax H3 VAE Load (B200 INT8)"}
