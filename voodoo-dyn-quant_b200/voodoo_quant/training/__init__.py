"""Training-step pieces of the B200 path (fused distillation loss)."""
