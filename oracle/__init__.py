"""CPU oracle for the paged KV-cache hot path: test infrastructure, not product code."""
