"""Validation suites, the operator benchmark and loop oracles."""
