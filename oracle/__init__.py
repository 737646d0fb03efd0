"""CPU oracle of the embedding-bag path (test infrastructure only)."""
