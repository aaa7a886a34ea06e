"""``krunch.inference`` is ``krunch_b200.inference`` (the same module object)."""
import sys

from krunch_b200 import inference as _impl

sys.modules[__name__] = _impl
