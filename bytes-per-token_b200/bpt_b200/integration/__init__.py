"""The seams where this package's kernels plug into the reference's engine (nanoserve):

- `paged_cache.PagedQuantizedKVCache`: a paged FP8 / INT8 KV cache with the `attend(layer, q, k, v, meta, scale)`
  seam of `src/fastserve/integration/kv_cache.py` (write through `quantize_kv_paged`, decode through the paged
  attention kernel);
- the W4A16 module swap is `bpt_b200.kernels.w4a16.install_w4a16` (the seam of `src/fastserve/quant/model.py`).
"""

from bpt_b200.integration.paged_cache import DecodeFn, OutOfBlocksError, PagedQuantizedKVCache, PagedQuantMeta

__all__ = ["DecodeFn", "OutOfBlocksError", "PagedQuantMeta", "PagedQuantizedKVCache"]
