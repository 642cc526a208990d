"""B200-native (sm_100a) Mamba-3 mixer: drop-in for jreoka/mamba3's ``Mamba3``."""

from .model import Mamba3

__all__ = ["Mamba3"]
