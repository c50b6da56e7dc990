"""NumPy stand-in for ``mlx`` used only to execute the reference's CPU path when building
golden fixtures; see ``mlx.core`` in this folder."""
