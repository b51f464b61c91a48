"""Atomic sharded checkpoints, validation and recovery."""
