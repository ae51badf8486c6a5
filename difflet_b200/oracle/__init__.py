"""CPU reference implementations (fp32 / fp64) used as test oracles."""
