"""Experiment launchers: executor pipelines and environment-variable arms."""
