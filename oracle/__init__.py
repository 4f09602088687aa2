"""CPU restatement of the TT-KV hot path (test infrastructure only: the checker, never the product)."""
