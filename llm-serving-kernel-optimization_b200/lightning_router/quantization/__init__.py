"""4-bit weight quantization and packing utilities."""
