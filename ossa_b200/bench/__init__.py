"""Model-integration helpers mirroring ``ossa.bench`` (patched attention forward)."""
