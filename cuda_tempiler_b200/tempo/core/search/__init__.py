"""Search space enumeration and build-free pruning."""
