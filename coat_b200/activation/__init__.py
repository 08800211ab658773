"""Activation-side operators of the hot path (mirror of coat/activation)."""
