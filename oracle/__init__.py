"""CPU oracle of the furnace reference decode path (test infrastructure only)."""
