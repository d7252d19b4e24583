"""Host-side allocator of the paged-KV path (``serve.block_manager``)."""
