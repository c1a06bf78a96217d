"""``metagross._C`` is ``metagross_b200._C`` (the same module object)."""
import sys

from metagross_b200 import _C as _impl

sys.modules[__name__] = _impl
