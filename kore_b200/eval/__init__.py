"""Evaluation: fast_p, matched-budget bake-off, paired statistics, stage and
retention gates, generalisation split checks, benchmark adapters."""
