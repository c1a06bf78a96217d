"""``metagross.attention`` is ``metagross_b200.attention`` (the same module object)."""
import sys

from metagross_b200 import attention as _impl

sys.modules[__name__] = _impl
