"""``krunch.chunking`` is ``krunch_b200.chunking`` (the same module object)."""
import sys

from krunch_b200 import chunking as _impl

sys.modules[__name__] = _impl
