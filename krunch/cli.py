"""``krunch.cli`` is ``krunch_b200.cli`` (the same module object)."""
import sys

from krunch_b200 import cli as _impl

sys.modules[__name__] = _impl
