"""Drop-in mirrors of the reference's opt/* entry points (fishelegs/ComfyUI-H3VAE-PyOpt 0.2.0).

Each module keeps the reference module's public names, argument order and meaning, and error
types (ValueError for contract violations, RuntimeError for platform/no-fallback failures), and
implements them with the sm_100a kernels of h3vae_b200.kernels.  Ops that the reference registers
with torch.library are registered here in the h3vae_b200_* namespaces with register_fake shape
functions.  The kernels are shape-generic where the reference pins the H3 shapes (width 2048,
B4 x 1797 tokens), so the same ops serve the BASELINE configs.
"""
