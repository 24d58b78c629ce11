"""Matched GPU / oracle models for the parity tests (built by oracle/pair.py)."""
from oracle.pair import build_pair, packed, rel_l2  # noqa: F401
