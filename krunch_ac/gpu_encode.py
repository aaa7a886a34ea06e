"""``krunch_ac.gpu_encode`` is ``krunch_b200.krunch_ac.gpu_encode`` (the same module object)."""
import sys

from krunch_b200.krunch_ac import gpu_encode as _impl

sys.modules[__name__] = _impl
