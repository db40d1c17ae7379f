"""CPU oracle of the DiffSpec draft-context path (test infrastructure only)."""
