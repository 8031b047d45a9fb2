"""Mamba-3 layer and decoder (same module layout as the reference's ``src/models``)."""

from src.models.mamba3 import Mamba3, MambaBlock, RMSNorm
from src.models.inference import Mamba3Decoder
