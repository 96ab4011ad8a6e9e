"""Transform calculus over kernel sources: typed exact / approximate
rewrites, the epsilon budget and relation lattice, the admissible action
space, and the opt-in self-extending library."""
from .budget import APPROX, EXACT, ErrorBudget, compose_eps, compose_relation, default_epsilon  # noqa: F401
from .calculus import Action, Transformation, admissible_actions, apply_sequence  # noqa: F401
from .library import APPROX_LIBRARY, EXACT_LIBRARY, LIBRARY, admissible, get_transform  # noqa: F401
