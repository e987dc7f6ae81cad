"""scacchi_b200: B200-native (sm_100a) batched Dirichlet-Thompson search step
with the public search/evaluator boundary of Francesco215/Scacchi."""

__version__ = "0.1.0"
