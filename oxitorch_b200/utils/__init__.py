"""Utilities mirroring the reference's ``oxitorch.utils`` package."""
