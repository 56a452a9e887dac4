"""jkb200 -- B200 (sm_100a) quantized-matmul hot path of jero-kernels-rvv.

The Python names mirror the public Rust API of the jero-kernels-rvv crate (quant_q8.rs,
quant.rs, repack.rs, ime.rs, lib.rs) so parity tests read like the crate's own tests. Every
call goes through the C ABI of include/jkb200.h in the in-tree libjkb200.so; there is no CPU
fallback. Device buffers are torch CUDA tensors (torch is only used for memory and streams).
"""
from .api import *  # noqa: F401,F403
from .api import __all__  # noqa: F401
