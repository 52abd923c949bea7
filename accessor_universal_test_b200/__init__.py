"""B200-native decode-fused DOT over compactly stored vectors.

The compute path is libautdot.so (CUDA, sm_100a) behind the C ABI in
include/autdot.h; C++ users include the headers in include/aut/ and link the
library.  This Python package is host plumbing over that C ABI:

* ``_lib``     -- ctypes binding (fails loudly when the library is missing);
* ``vectors``  -- device buffers of encoded vectors (torch for memory only);
* ``sharded``  -- contiguous sharding over GPUs with one FP64 all-reduce;
* ``build``    -- the nvcc build recipe.
"""
from ._lib import (  # noqa: F401
    ACC_FP32, ACC_FP64, DENSE, PADDED, TARGET_FP32, TARGET_FP64,
    AutError, Workspace, check, format_id, format_info, generate, load,
    storage_bytes,
)

# Formats with a fused DOT kernel, in the order of include/autdot.h.
DOT_FORMATS = ("fp32", "fp64", "e2m3", "e8m0", "e8m1", "e8m3", "e8m5",
               "bf16_e8m7", "e8m15", "lns8_r3", "lns16_r11")
