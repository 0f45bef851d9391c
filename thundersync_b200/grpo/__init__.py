"""GRPO: configuration, the reward-linear streaming objective and its DP trainer."""
