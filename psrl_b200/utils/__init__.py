"""Runtime utilities: events, profiling, checkpointing, RPC, concurrency."""
