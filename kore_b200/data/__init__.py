"""Data layer: tokenizers, chat templates, JSONL datasets and record schemas,
the data factory (generators, assembly, hygiene)."""
