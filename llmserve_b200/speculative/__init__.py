"""Speculative decoding (EAGLE3): result types, acceptance rules, fixed trees."""
