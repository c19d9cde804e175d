"""Serving: KV-cache generation engine and an HTTP API over it."""
