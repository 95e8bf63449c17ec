"""Host-side helpers around the drop-in rasterizer: synthetic scenes, the view-parallel
training step and its distributed plumbing."""
