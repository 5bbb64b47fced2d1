"""`import f16acc`: the reference's import name for this build.

steppergg/f16acc exposes `f16acc.mm`, `enable`, `disable` and `calls`
(f16acc/__init__.py:8-11) and its tests import `f16acc` and `from f16acc
import patch` (tests/test_f16acc.py:5-6).  This package gives exactly those
names, bound to the same objects as f16acc_b200's: `f16acc.patch` and
`f16acc.kernel` are the modules f16acc_b200.patch and f16acc_b200.kernel, so
`f16acc.calls is f16acc.patch.calls` and enable/disable swap the same
`torch.nn.functional.linear`.  Nothing is reimplemented here.
"""

import sys

from f16acc_b200 import calls, disable, enable, kernel, mm, patch

__all__ = ["mm", "enable", "disable", "calls"]

# `import f16acc.patch` / `import f16acc.kernel` resolve to the same module objects.
sys.modules[__name__ + ".patch"] = patch
sys.modules[__name__ + ".kernel"] = kernel
