"""Wire formats and signed control records."""
