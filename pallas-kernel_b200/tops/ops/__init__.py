"""Operators (reference ``tops/ops``)."""
