"""Transform calculus over kernel sources (exact and approximate rewrites)."""
