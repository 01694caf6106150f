"""CPU oracle of the reference GSA forward (test infrastructure; never imported by the product)."""
