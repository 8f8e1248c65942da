"""Research extensions (Flow-GRPO for flow-matching generators)."""
