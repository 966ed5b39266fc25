"""chunkkv_b200 — B200-native (sm_100a) blend prefill with the chunkkv Python API.

Modules mirror the reference package layout: engine.base / engine.torch_engine,
scheduler.rerope, store.keys / store.kvstore, types.  The compute runs in the
in-tree CUDA library libchunkkv_b200.so (C ABI in include/chunkkv_b200.h).
"""

__version__ = "0.1.0"
