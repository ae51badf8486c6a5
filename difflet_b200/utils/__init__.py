"""Runtime utilities: errors, timing, logging, environment."""
