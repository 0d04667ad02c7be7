"""GLM-5.2 MoE-block constants and benchmark regimes (glm52/config.py:15-89).

Values are the model's (zai-org/GLM-5.2 config.json as recorded by the reference); only
the ones on the MoE-block path are kept.
"""

from __future__ import annotations

from dataclasses import dataclass

HIDDEN_SIZE = 6144
MOE_INTERMEDIATE_SIZE = 2048
N_ROUTED_EXPERTS = 256
N_SHARED_EXPERTS = 1
NUM_EXPERTS_PER_TOK = 8
ROUTED_SCALING_FACTOR = 2.5
NORM_TOPK_PROB = True
SCORING_FUNC = "sigmoid"
TOPK_METHOD = "noaux_tc"
N_GROUP = 1
TOPK_GROUP = 1
RMS_NORM_EPS = 1e-5
# o_proj contraction width (glm52/config.py:55-59): absorbed MLA at decode emits
# [T, heads, kv_lora_rank], non-absorbed MLA at prefill [T, heads, v_head_dim]
OPROJ_K_DECODE = 64 * 512  # 32768
OPROJ_K_PREFILL = 64 * 256  # 16384
W13_N = 2 * MOE_INTERMEDIATE_SIZE
W2_K = MOE_INTERMEDIATE_SIZE


@dataclass(frozen=True)
class Regime:
    """One benchmark point: T tokens through one MoE block."""

    name: str
    T: int

    @property
    def moe_rows(self) -> int:
        return self.T * NUM_EXPERTS_PER_TOK


DECODE_REGIMES = [Regime(f"decode_bs{t}", t) for t in (1, 8, 32, 64, 128, 256)]
PREFILL_REGIMES = [Regime(f"prefill_t{t}", t) for t in (2048, 4096, 8192)]
ALL_REGIMES = DECODE_REGIMES + PREFILL_REGIMES
BASELINE_T = (1, 32, 256, 2048, 8192)
