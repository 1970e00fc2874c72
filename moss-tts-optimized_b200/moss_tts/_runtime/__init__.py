"""Decode runtime: C-ABI bindings, operator wrappers, weights and the decode engine."""
