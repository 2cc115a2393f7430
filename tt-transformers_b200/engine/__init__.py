"""The engine: the step function, the scheduler above it, and the Python entry point."""
