"""Measurement utilities (not on the transform path)."""
