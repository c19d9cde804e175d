"""Blackwell-native (sm_100a) MoE language-model training framework."""

__version__ = "0.1.0"
