"""Import name of the reference package (``krunch``) mapped onto krunch_b200.

``import krunch.inference``, ``from krunch.chunking import compress_all``,
``krunch.batched_rwkv4``, ``krunch.cpp_path``, ``krunch.cli`` and
``krunch.job`` resolve to the krunch_b200 modules themselves (the same module
objects), so the reference's callers run unchanged on this build.
"""
