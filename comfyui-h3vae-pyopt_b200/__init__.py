"""ComfyUI custom-node directory for the B200-native H3 video VAE.

ComfyUI loads a custom-node directory by executing its __init__.py as a flat module, so this
file puts its own directory on sys.path and imports the node mappings from h3vae_b200.nodes.
"""
import os
import sys

__version__ = "0.1.0"

_here = os.path.dirname(os.path.realpath(__file__))
if _here not in sys.path:
    sys.path.insert(0, _here)

from h3vae_b200.nodes import NODE_CLASS_MAPPINGS, NODE_DISPLAY_NAME_MAPPINGS  # noqa: E402

__all__ = ["NODE_CLASS_MAPPINGS", "NODE_DISPLAY_NAME_MAPPINGS"]
