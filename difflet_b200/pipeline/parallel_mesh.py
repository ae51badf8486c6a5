"""Re-export of the mesh math under the reference's module path."""

from difflet_b200.parallel.mesh import AXES, MeshCoords, MeshSpec  # noqa: F401
