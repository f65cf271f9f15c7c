"""Shared chunk-state scans (reference ``tops/ops/common``)."""
