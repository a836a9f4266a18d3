"""Test-only stand-in for the Emmy IR package (see emmy/_core.py)."""
