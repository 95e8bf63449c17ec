from .rasterize import RasterizeFunction, rasterize

__all__ = ["RasterizeFunction", "rasterize"]
