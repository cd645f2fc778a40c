"""B200-native (sm_100a) RACE attention: drop-in for the reference's
BatchedACE / RACEAttention / RACEBlock modules.

    from race_attention_b200 import race_attention          # autograd op
    from race_attention_b200.vit import RACEAttention        # non-causal
    from race_attention_b200.race import RACEAttention       # causal
"""
from .functional import race_attention  # noqa: F401

__all__ = ["race_attention"]
