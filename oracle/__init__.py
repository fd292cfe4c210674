"""CPU oracle of the exact k-NN hot path: test infrastructure, not product."""
