"""ComfyUI custom node: ZImage Triton Accelerate on B200 (sm_100a kernels).

Registers the same node class and display name as the reference
(__init__.py:16-22 of newgrit1004/ComfyUI-ZImage-Triton).
"""

import os
import sys

_here = os.path.dirname(os.path.abspath(__file__))
if _here not in sys.path:
    sys.path.insert(0, _here)

try:
    from .nodes import ZImageTritonApply
except ImportError:  # loaded outside a package (e.g. by path)
    from nodes import ZImageTritonApply  # type: ignore[no-redef]

NODE_CLASS_MAPPINGS = {
    "ZImageTritonApply": ZImageTritonApply,
}
NODE_DISPLAY_NAME_MAPPINGS = {
    "ZImageTritonApply": "ZImage Triton Accelerate",
}

__all__ = ["NODE_CLASS_MAPPINGS", "NODE_DISPLAY_NAME_MAPPINGS"]
