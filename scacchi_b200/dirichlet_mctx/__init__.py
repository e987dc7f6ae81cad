"""B200 implementation of the Dirichlet-Thompson tree search
(``scacchi.dirichlet_mctx`` of Francesco215/Scacchi): same public names, the
tree on the GPU, every phase a CUDA kernel."""

from .base import PolicyOutput, RecurrentFnOutput, RootFnOutput
from .policies import dirichlet_thompson_policy
from .posterior_updates import update_posterior, update_posterior_prefix_cdf
from .prefix_cdf import BinaryPrefixQuadraturePolicy, binary_posterior_best_policy_prefix_quadrature
from .tree import (ChildrenView, LeafView, NodeView, PosteriorUpdate, PosteriorUpdateContext, SearchSummary, Tree,
                   instantiate_tree_from_root)

__all__ = [
    "BinaryPrefixQuadraturePolicy", "ChildrenView", "LeafView", "NodeView", "PolicyOutput", "PosteriorUpdate",
    "PosteriorUpdateContext", "RecurrentFnOutput", "RootFnOutput", "SearchSummary", "Tree",
    "binary_posterior_best_policy_prefix_quadrature", "dirichlet_thompson_policy", "instantiate_tree_from_root",
    "update_posterior", "update_posterior_prefix_cdf",
]
