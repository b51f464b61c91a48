"""Step logic, optimizers, schedule and the trainer."""
