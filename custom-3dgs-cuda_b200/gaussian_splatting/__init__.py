"""Python side of the drop-in: the `gaussian_splatting.rasterizer` wrapper and the scene
containers it type-checks against, with the reference's module paths."""
