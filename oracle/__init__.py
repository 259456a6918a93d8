"""CPU oracle and CPU baseline for the paged-KV path (test infrastructure only)."""
