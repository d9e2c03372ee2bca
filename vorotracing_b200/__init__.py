"""B200-native Voronoi ray traversal (VoroTracing hot path)."""
__version__ = "0.1.0"
