"""Runtime: training engine, paged inference, checkpoints, planning, metrics, faults."""
