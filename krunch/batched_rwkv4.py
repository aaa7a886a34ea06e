"""``krunch.batched_rwkv4`` is ``krunch_b200.batched_rwkv4`` (the same module object)."""
import sys

from krunch_b200 import batched_rwkv4 as _impl

sys.modules[__name__] = _impl
