"""The ownership map of sequence-sharded steps (tritiercache_b200/csrc/tt_attn.cuh:
shard_map, dense_local_slot, packed_global, ring_slot_id), checked on the host.

tests/shard_map_check.cu includes the library's own header and, for 4000
random tier layouts and world sizes 1..8, checks that the ranks' local
positions cover every sink, heavy-hitter and ring slot and every packed token
exactly once, that ownership follows its rule (slot j on rank j % world,
256-token granule k on rank k % world), that each rank's packed tokens are in
granule order, and that the ring slots' token ids are exactly
[total - n2, total) (in logical order when unsharded).  It also checks the
float order keys (order_key / key_value) behind the threshold's radix select
and the routing rows' complemented (score, slot) minimum.  nvcc builds it as a
host program; no GPU is used.
"""
import os
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def test_ownership_map_partitions_every_tier(tmp_path):
    if not os.path.exists(NVCC):
        pytest.skip("nvcc not available")
    exe = str(tmp_path / "shard_map_check")
    subprocess.run([NVCC, "-std=c++17", "-O1", "-gencode", "arch=compute_100a,code=sm_100a", "-o", exe,
                    os.path.join(HERE, "shard_map_check.cu")], check=True,
                   capture_output=True, timeout=300)
    out = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and out.stdout.startswith("ok"), out.stdout + out.stderr
