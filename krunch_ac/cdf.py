"""``krunch_ac.cdf`` is ``krunch_b200.krunch_ac.cdf`` (the same module object)."""
import sys

from krunch_b200.krunch_ac import cdf as _impl

sys.modules[__name__] = _impl
