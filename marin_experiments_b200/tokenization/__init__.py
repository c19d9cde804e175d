"""Tokenizer training (plain BPE, SuperBPE) and the tokenizer bake-off cost model."""
