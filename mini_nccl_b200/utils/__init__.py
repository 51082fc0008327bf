"""Utilities: device timing, clock sampling, environment helpers."""
