"""kore_b200: a B200-native (sm_100a) post-training framework with KORE's
capabilities: SFT / midtrain / DPO / multi-turn GRPO trainers, a rollout
engine, and a verified kernel environment with a roofline reward."""
__version__ = "0.1.0"
