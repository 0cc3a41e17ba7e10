"""B200-native drop-in for rust-llm-pager's ``pager_hf`` decode-attention hot path.

``streaming_attention`` keeps the reference module's public functions and adds
the fused block-table op; ``kv_block_store`` holds KV blocks in a device pool
and a pinned host pool.  The compute is in ``libpager_b200.so`` (C ABI,
include/pager_b200.h).
"""
