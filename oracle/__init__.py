"""CPU oracle of the 3D deformable slide attention hot path (test infrastructure only)."""
