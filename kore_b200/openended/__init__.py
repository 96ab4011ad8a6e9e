"""Open-ended co-evolution curriculum: SELECT tasks at the policy's frontier
(learnability, regret, novelty over a MAP-Elites archive) and MINT new
correct-by-construction tasks from a typed grammar."""
