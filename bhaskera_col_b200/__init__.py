"""B200-native (sm_100a) TurboQuant KV-cache path for bhaskera-infer.

Public surface mirrors bhaskera.inference.kv_cache; see
``bhaskera_col_b200.inference.kv_cache``.
"""
__version__ = "0.1.0"
