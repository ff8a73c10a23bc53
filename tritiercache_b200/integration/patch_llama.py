"""Re-export of the universal patcher under the reference's legacy module name
(src/tri_tier/integration/patch_llama.py:7-37)."""
from .patch_model import (H_RATIO, HAS_CPP_EXT, K_GROUP_SIZE, MAX_SEQ_LEN, PBS_METADATA_DTYPE, R_SIZE, SCORE_DECAY,
                          _reference_attention_path, apply_patch, is_patched, patched_forward, remove_patch,
                          reset_caches)

__all__ = ["apply_patch", "remove_patch", "reset_caches", "is_patched", "patched_forward",
           "_reference_attention_path", "MAX_SEQ_LEN", "R_SIZE", "H_RATIO", "SCORE_DECAY", "K_GROUP_SIZE",
           "PBS_METADATA_DTYPE", "HAS_CPP_EXT"]
