"""Training data on disk: cdl's token cache format and a device loader."""

from cdl_b200.data.token_cache import (CACHE_FORMAT, BlockDataset, CacheMeta, DeviceBlockLoader, TokenCache,
                                       build_from_tokens, token_dtype)

__all__ = ["CACHE_FORMAT", "BlockDataset", "CacheMeta", "DeviceBlockLoader", "TokenCache", "build_from_tokens",
           "token_dtype"]
