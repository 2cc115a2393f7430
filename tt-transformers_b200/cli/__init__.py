"""Command lines: demo (generate from a prompt) and benchmark (--case ...)."""
