"""Source admission and cross-rank work claims (host side)."""
