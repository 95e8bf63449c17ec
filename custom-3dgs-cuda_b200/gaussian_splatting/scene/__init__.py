from .camera import camera
from .gaussian import gaussian

__all__ = ["camera", "gaussian"]
