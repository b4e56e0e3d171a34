"""pagellm_b200: pagellm's paged KV-cache hot path on B200 (sm_100a).

``pagellm_b200.cache`` keeps the API of ``pagellm.cache.paged``; the work runs in
libpagekv.so (CUDA kernels behind a C ABI, ``include/pagekv.h``), built in-tree by
``python -m pagellm_b200.build``.
"""

__version__ = "0.1.0"
