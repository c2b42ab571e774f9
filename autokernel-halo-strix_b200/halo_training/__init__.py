"""124M hybrid LM and its data-parallel training step (the end-to-end measurement)."""
