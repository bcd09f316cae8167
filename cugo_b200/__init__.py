"""cugo_b200: B200-native batch environment for Hangame Shin Matgo self-play.

    from cugo_b200 import load_extension
    ext = load_extension()          # same ops as the reference's cugo_torch50_ext
"""
from .ext import CugoB200Extension, load_extension, load_library

__all__ = ["CugoB200Extension", "load_extension", "load_library"]
