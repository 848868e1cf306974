"""Research experiment recipes."""
