"""B200-native H3 video-VAE INT8 encode/decode path (sm_100a kernels behind a C ABI).

Submodules:
  kernels   tensor-level wrappers of every C entry point (libh3vae_b200.so)
  opt       drop-in mirrors of the reference's opt/* entry points
  model     H3-structured encoder/decoder assembled from those kernels
  runtime   H3VAEPyOptRuntime (ComfyUI first_stage_model) and tile scheduling
  nodes     the H3VAEPyOptLoader ComfyUI node
"""
__version__ = "0.1.0"
