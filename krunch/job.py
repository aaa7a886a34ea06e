"""``krunch.job`` is ``krunch_b200.job`` (the same module object)."""
import sys

from krunch_b200 import job as _impl

sys.modules[__name__] = _impl
