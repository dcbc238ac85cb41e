"""Parity checkers for the MoE FFN path (test infrastructure, not product code)."""
