"""CPU oracle of the paged-decode path (test infrastructure only; never imported by the product)."""
