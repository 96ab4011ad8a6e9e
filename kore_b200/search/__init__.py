"""AlphaKernel value-guided search over verified kernel rewrites."""
from .alphakernel import AlphaKernel, Eval, RooflineCeiling, SearchResult, fingerprint, make_roofline_ub_fn, search  # noqa: F401
from .bandit import Budget, MeasureStats, successive_halving  # noqa: F401
from .propose import TransformProposePolicy, search_from_kernel  # noqa: F401
