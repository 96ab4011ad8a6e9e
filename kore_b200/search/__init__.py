"""Test-time kernel search: bandits and best-first / PUCT search over transforms."""
