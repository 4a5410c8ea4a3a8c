"""Serving-core contracts kept API-compatible with Artifex-Assistant v5 (core/ in the reference)."""
