"""larynx_b200: the Flow decoder hot path of hardenedlinux/larynx (22-block DiT
estimator inside the 10-step CFG CFM Euler loop) as hand-written sm_100a CUDA
behind a C ABI (include/larynx_flow.h).  This package is the Python host side:
a ctypes binding (flow.py) and the GGUF / noise-asset writers (gguf.py)."""

from .flow import FlowDecoder, FlowError, load_library, LIB_PATH, EXPORTS  # noqa: F401
