"""cacheflow_b200: B200-native (sm_100a) KV-cache kernel layer with CacheFlow's operator API.

The compute lives in libcacheflow_b200.so (CUDA C++, built in-tree by
`python -m cacheflow_b200.build`); this package only binds it (ctypes) and
provides torch-tensor conveniences, the decode-step engine and the multi-GPU
sequence sharding.
"""

from ._lib import CacheFlowError, load  # noqa: F401

__version__ = "0.1.0"
