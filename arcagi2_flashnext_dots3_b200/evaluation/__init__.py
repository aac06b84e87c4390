"""Evaluation tooling: task scoring and budget-limited solver simulation, paired bootstrap comparison of two
builds, teacher-forced KL fidelity between two models, degeneration checks and leaf-wise build comparison."""
