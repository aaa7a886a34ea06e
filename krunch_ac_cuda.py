"""Import name of the reference's native extension ``krunch_ac_cuda``
(krunch_ac/cuda/main.cpp:354-466, layer_cpp.cpp:824-1053) mapped onto
krunch_b200.krunch_ac_cuda (the same module object): coder, CDF, GEMM and
layer-step entry points with the reference's tensor contracts."""
import sys

from krunch_b200 import krunch_ac_cuda as _impl

sys.modules[__name__] = _impl
