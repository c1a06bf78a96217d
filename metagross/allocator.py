"""``metagross.allocator`` is ``metagross_b200.allocator`` (the same module object)."""
import sys

from metagross_b200 import allocator as _impl

sys.modules[__name__] = _impl
