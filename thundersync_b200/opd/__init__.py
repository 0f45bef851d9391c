"""On-policy distillation objectives."""
