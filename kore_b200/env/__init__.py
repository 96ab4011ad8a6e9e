"""Environments: the verified kernel environment (KoreEnv), its replay cache,
and the synthetic benchmark environment."""
