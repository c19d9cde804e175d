"""Reinforcement learning on generated completions: GRPO / Dr.GRPO, environments, learner."""
