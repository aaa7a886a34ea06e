"""``krunch.cpp_path`` is ``krunch_b200.cpp_path`` (the same module object)."""
import sys

from krunch_b200 import cpp_path as _impl

sys.modules[__name__] = _impl
