"""adai_b200 — B200-native (sm_100a) batched KV-cached decode step of the kerfbit/adai
encoder-decoder, behind a C ABI (include/adai_b200.h, libadai_b200.so).

Python here is a thin ctypes binding for tests and benchmarks; the product is the shared
library built from adai_b200/csrc.
"""
from .config import ModelConfig, Workload, WORKLOADS, TINY, MID, LARGE  # noqa: F401
from .api import Context, KVArena, load, EXPORTS  # noqa: F401
