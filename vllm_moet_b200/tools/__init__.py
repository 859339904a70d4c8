"""Offline studies and utilities (not on the serving path)."""
