"""Drafters and their model-specific objectives (reference layout: models/<name>/)."""
