"""nspeech_b200 -- B200-native (sm_100a) GGUF Q8_0 contraction library.

Host-side mirror of nspeech's Q8_0 matmul path over the C ABI of
``libnq8.so`` (include/nq8.h):

* ``fast_matmul``  -- ``MatMul`` / ``QWeight`` (src/fast_matmul.rs)
* ``dispatch``     -- named entry points of src/triton_kernels.rs
* ``lib``          -- ctypes binding, status codes, error type
"""
from .lib import NqError, init  # noqa: F401

__all__ = ["NqError", "init"]
