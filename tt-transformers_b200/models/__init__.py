"""Architectures: each module turns its typed configuration into a ModelSpec."""
