"""Camera container with the reference's field names (gaussian_splatting/scene/camera.py:3-38):
world-to-camera R[N,3,3] and t[N,3], pinhole intrinsics fx, fy, cx, cy as [N,1]."""

import torch


class camera:  # noqa: N801 - reference class name
    def __init__(self, N: int) -> None:
        self.N = N
        self.R = torch.zeros(N, 3, 3, dtype=torch.float32)
        self.t = torch.zeros(N, 3, dtype=torch.float32)
        self.fx = torch.zeros(N, 1, dtype=torch.float32)
        self.fy = torch.zeros(N, 1, dtype=torch.float32)
        self.cx = torch.zeros(N, 1, dtype=torch.float32)
        self.cy = torch.zeros(N, 1, dtype=torch.float32)

    def sample_camera_view(self) -> list[dict]:
        """One view dict per camera (keys R, T, fx, fy, cx, cy, image_path, image_name)."""
        paths = getattr(self, "image_paths", [None] * self.N)
        names = getattr(self, "image_names", [None] * self.N)
        return [
            {"R": self.R[i], "T": self.t[i], "fx": self.fx[i], "fy": self.fy[i],
             "cx": self.cx[i], "cy": self.cy[i], "image_path": paths[i], "image_name": names[i]}
            for i in range(self.N)
        ]
