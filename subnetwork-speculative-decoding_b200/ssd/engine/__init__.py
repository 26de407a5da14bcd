from ssd.engine.kv_cache import KVCache

__all__ = ["KVCache"]
