"""Campaign orchestration: staged pipeline with a resumable manifest, the
process supervisor, and shared-node helpers (free-GPU picking, LPT work
partitioning)."""
