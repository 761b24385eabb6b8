"""CPU oracle for the DoRA hot path (test infrastructure; never imported by the product)."""
