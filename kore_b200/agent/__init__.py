"""Agentic tool harness: multi-turn tool-use loop over the kernel environment."""
