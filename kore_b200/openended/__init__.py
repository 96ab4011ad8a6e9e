"""Open-ended task curriculum: task space, MAP-Elites archive, proposer,
controller, coevolution loop, task minter."""
