"""B200-native (sm_100a) chunk-causal cached attention for Hy-Nomas.

Public surface (mirrors the reference's names):
  * ``causal_attention_with_cache_mp``  drop-in for hymm/models/dit/nomas_cpt.py:335
  * ``kv_cache``        INT8 / E4M3 cache storage (int8_kv_cache.py, kv_cache_storage.py)
  * ``communications``  Ulysses exchange (hymm/distributed/communications.py)
  * ``ring``            ring (KV-passing) sequence parallelism with LSE merge
  * ``window``          sink + sliding-window history selection
  * ``install``         monkey-patch installer for a running reference process
The kernels live in ``libhyb200.so`` (``include/hyb200.h``), built by ``build.py``.
"""
from . import _lib, kv_cache, parallel_states  # noqa: F401
from .attention import causal_attention_with_cache_mp, cached_attention_local  # noqa: F401

__all__ = ["causal_attention_with_cache_mp", "cached_attention_local", "kv_cache", "parallel_states"]
