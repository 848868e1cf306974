"""Shell recipes (validation, smoke, benchmarks, experiments) and their report helpers."""
