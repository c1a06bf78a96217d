"""The reference's import path, served by this repository's B200 path.

``import metagross``, ``from metagross import _C``, ``metagross.allocator``,
``metagross.cache`` and ``metagross.attention`` resolve to the modules of
``metagross_b200`` (each submodule here replaces itself with its counterpart
in ``sys.modules``), so code and tests written against the reference's Python
surface for the paged KV cache and decode attention run unchanged.  Only the
hot-path modules exist; the reference's Hugging Face generation and
perplexity modules (metagross/generate*.py, metagross/perplexity.py) are not
part of this path.
"""
from metagross_b200 import __version__, sanity_add  # noqa: F401
