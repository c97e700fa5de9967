"""Parity checkers for the FlashLog hot path (test infrastructure only).

The product (flashlog_b200) never imports this package.
"""
