"""See the package docstring of ``qwen35_b200``."""
