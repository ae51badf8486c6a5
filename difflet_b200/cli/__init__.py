"""Command-line interface (``python -m difflet_b200 ...``, console script ``difflet``)."""
