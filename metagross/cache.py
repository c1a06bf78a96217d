"""``metagross.cache`` is ``metagross_b200.cache`` (the same module object)."""
import sys

from metagross_b200 import cache as _impl

sys.modules[__name__] = _impl
