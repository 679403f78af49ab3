"""B200 (sm_100a) DeepSeek sparse-attention operator path.

Drop-in replacements for the three operators of zhutianci/ascendc_kernel:

* :mod:`ascendc_kernel_b200.sparse_attn` -- SparseAttention (Task 1)
* :mod:`ascendc_kernel_b200.indexer`     -- Lightning Indexer (Task 2)
* :mod:`ascendc_kernel_b200.sinkhorn`    -- Sinkhorn / mHC (Task 3)

Each module keeps the reference's ``ModelNew`` / ``get_inputs`` /
``get_init_inputs`` interface; the compute is the in-tree CUDA library
``lib/libdsa_b200.so`` (C ABI: ``include/dsa_b200.h``), loaded lazily.
"""

__version__ = "0.1.0"
