from .triangle import FastTriangleMultiplication  # noqa: F401
