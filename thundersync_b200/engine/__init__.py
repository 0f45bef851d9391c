"""Execution core: segment forests, plans, the streaming executor, sharded steps."""
