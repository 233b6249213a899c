"""NoriCausal: zero-shot causal graph estimation from one table (reference ``src/synthefy_nori/causal``)."""

from synthefy_nori_b200.causal.estimator import NoriCausal, get_decoded_graph
from synthefy_nori_b200.causal.network import NoriCausalNetwork
from synthefy_nori_b200.causal.registry import NORI_CAUSAL_MODELS

__all__ = ["NoriCausal", "NoriCausalNetwork", "NORI_CAUSAL_MODELS", "get_decoded_graph"]
