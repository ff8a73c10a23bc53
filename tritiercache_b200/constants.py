"""Constants of the reference package (src/tri_tier/constants.py:1-7).

DEVICE is "cuda": the tiers live in HBM and every kernel runs on the GPU.
"""
DEVICE = "cuda"

UPDATE_THRESHOLD = 32

CHUNK_SIZE = 16

SINK_SIZE = 4
