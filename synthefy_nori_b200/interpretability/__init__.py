"""Model explanations for a fitted ``NoriRegressor`` (reference ``src/synthefy_nori/interpretability``):
Shapley attributions by feature imputation, partial dependence / ICE, sequential feature
selection, glass-box distillation and the one-call ``NoriInterpreter``.  Every explainer batches all of its perturbed rows
into one query block, so an explanation is one pass of the cached context."""

from synthefy_nori_b200.interpretability.feature_selection import FeatureSelectionResult, feature_selection
from synthefy_nori_b200.interpretability.glassbox import GlassBoxModel, distill_glassbox
from synthefy_nori_b200.interpretability.interpreter import NoriInterpreter
from synthefy_nori_b200.interpretability.pdp import partial_dependence, partial_dependence_plots
from synthefy_nori_b200.interpretability.shapley import ImputationExplainer, get_nori_imputation_explainer

__all__ = ["NoriInterpreter", "FeatureSelectionResult", "feature_selection", "GlassBoxModel", "distill_glassbox", "partial_dependence",
           "partial_dependence_plots", "ImputationExplainer", "get_nori_imputation_explainer"]
