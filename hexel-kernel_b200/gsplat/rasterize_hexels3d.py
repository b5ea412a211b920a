"""3D Hexel surfel rasteriser (filled in below)."""

__all__: list = []
