"""Equivalence oracle: random trials, adversarial battery, metamorphic
relations and determinism, combined into one verdict."""
