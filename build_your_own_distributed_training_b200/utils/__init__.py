"""Launch environment, dtype policy and RNG helpers."""
