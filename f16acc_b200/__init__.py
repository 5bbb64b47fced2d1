"""B200-native (sm_100a) chunked FP16-accumulate GEMM with the drop-in API of
steppergg/f16acc (f16acc/__init__.py:8-11): `mm`, `enable`, `disable`, `calls`.

Each 32-long K chunk is accumulated in FP16 on the tensor cores and the chunks
are added in FP32; tiles whose FP16 chunk overflowed are redone with FP32
accumulation on the device, with no host sync.
"""

from .kernel import mm
from .patch import calls, disable, enable

__all__ = ["mm", "enable", "disable", "calls"]
