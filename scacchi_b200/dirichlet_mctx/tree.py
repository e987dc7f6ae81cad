"""Device-resident search tree (tree.py of the reference).

The tree is one struct-of-arrays workspace on the GPU (layout documented in
include/scacchi_b200.h).  Action rows are padded to a multiple of 32 so a
warp reads a row with aligned 32-wide accesses; the attributes below expose
the reference's field names as views trimmed to the real action count.

Embeddings: any pytree of tensors with a leading batch axis (tensor, dict,
list, tuple, NamedTuple).  It is packed into one byte row per node so the
kernels can gather a parent's embedding and store a child's without knowing
its structure.
"""

from __future__ import annotations

import ctypes as C
import dataclasses
import math
from typing import Any

import torch

from .. import _lib
from .outcomes import NO_DISTANCE, NO_OUTCOME

ROW_ALIGN = 32


def action_stride(num_actions: int) -> int:
    return ((num_actions + ROW_ALIGN - 1) // ROW_ALIGN) * ROW_ALIGN


def stream_handle(device: torch.device) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def ptr(t: torch.Tensor | None) -> C.c_void_p | None:
    if t is None:
        return None
    return C.c_void_p(t.data_ptr())


# --------------------------------------------------------------------------
# embedding codec
# --------------------------------------------------------------------------

def _flatten(tree: Any):
    if tree is None:
        return [], lambda leaves: None
    if isinstance(tree, torch.Tensor):
        return [tree], lambda leaves: leaves[0]
    if isinstance(tree, dict):
        keys = list(tree.keys())
        parts = [_flatten(tree[k]) for k in keys]
        sizes = [len(p[0]) for p in parts]

        def rebuild(leaves):
            out, i = {}, 0
            for k, (_, rb), n in zip(keys, parts, sizes):
                out[k] = rb(leaves[i:i + n])
                i += n
            return out
        return [l for p in parts for l in p[0]], rebuild
    if isinstance(tree, (list, tuple)):
        parts = [_flatten(v) for v in tree]
        sizes = [len(p[0]) for p in parts]
        is_named = hasattr(tree, "_fields")

        def rebuild(leaves):
            vals, i = [], 0
            for (_, rb), n in zip(parts, sizes):
                vals.append(rb(leaves[i:i + n]))
                i += n
            if is_named:
                return type(tree)(*vals)
            return type(tree)(vals)
        return [l for p in parts for l in p[0]], rebuild
    raise TypeError(f"unsupported embedding leaf type {type(tree)!r}")


class EmbeddingCodec:
    """Packs a batched pytree of tensors into uint8 rows [..., nbytes]."""

    def __init__(self, example: Any):
        leaves, self._rebuild = _flatten(example)
        self.specs = []
        off = 0
        for leaf in leaves:
            shape = tuple(leaf.shape[1:])
            n = int(math.prod(shape)) * leaf.element_size()
            self.specs.append((off, n, leaf.dtype, shape))
            off += (n + 7) // 8 * 8
        self.nbytes = off

    def pack(self, tree: Any, batch: int, device) -> torch.Tensor:
        buf = torch.zeros((batch, max(self.nbytes, 1)), dtype=torch.uint8, device=device)
        leaves, _ = _flatten(tree)
        for (off, n, dtype, shape), leaf in zip(self.specs, leaves):
            if n == 0:
                continue
            rows = leaf.to(device=device, dtype=dtype).reshape(batch, -1).contiguous()
            buf[:, off:off + n] = rows.view(torch.uint8).reshape(batch, n)
        return buf[:, :self.nbytes] if self.nbytes else buf[:, :0]

    def unpack(self, buf: torch.Tensor) -> Any:
        lead = tuple(buf.shape[:-1])
        leaves = []
        for off, n, dtype, shape in self.specs:
            raw = buf[..., off:off + n].contiguous()
            leaves.append(raw.view(dtype).reshape(*lead, *shape))
        return self._rebuild(leaves)


# --------------------------------------------------------------------------
# tree
# --------------------------------------------------------------------------

@dataclasses.dataclass(frozen=True)
class SearchSummary:
    """tree.py:86-98."""

    visit_counts: torch.Tensor
    alpha: torch.Tensor
    value_alpha: torch.Tensor
    q_categorical_outcome: torch.Tensor
    q_categorical_distance: torch.Tensor
    v_categorical_outcome: torch.Tensor
    v_categorical_distance: torch.Tensor


class Tree:
    """Fixed-capacity tree [B, num_nodes, ...] (tree.py:140-242)."""

    ROOT_INDEX = 0
    NO_PARENT = -1
    UNVISITED = -1

    def __init__(self, batch: int, num_nodes: int, num_actions: int, codec: EmbeddingCodec | None = None,
                 device: torch.device | str | None = None):
        if not 1 <= num_actions <= 128:
            raise ValueError(f"num_actions must be in [1, 128], got {num_actions}")
        self.device = torch.device(device if device is not None else "cuda")
        self.batch, self.capacity, self.A = int(batch), int(num_nodes), int(num_actions)
        self.S = action_stride(num_actions)
        self.codec = codec
        self.E = codec.nbytes if codec is not None else 0
        B, Cn, S, dev = self.batch, self.capacity, self.S, self.device
        i32, i8, f32, u8 = torch.int32, torch.int8, torch.float32, torch.uint8
        self.parents_ = torch.empty((B, Cn), dtype=i32, device=dev)
        self.children_ = torch.empty((B, Cn, S), dtype=i32, device=dev)
        self.to_play_ = torch.empty((B, Cn), dtype=i32, device=dev)
        self.node_outcome_ = torch.empty((B, Cn), dtype=i8, device=dev)
        self.node_payload_ = torch.empty((B, Cn), dtype=i32, device=dev)
        self.edge_outcome_ = torch.empty((B, Cn, S), dtype=i8, device=dev)
        self.edge_payload_ = torch.empty((B, Cn, S), dtype=i32, device=dev)
        self.value_prior_ = torch.empty((B, Cn, 2), dtype=f32, device=dev)
        self.value_alpha_ = torch.empty((B, Cn, 2), dtype=f32, device=dev)
        self.edge_alpha_ = torch.empty((B, Cn, S, 2), dtype=f32, device=dev)
        self.invalid_ = torch.empty((B, Cn, S), dtype=u8, device=dev)
        self.embedding_ = torch.empty((B, Cn, max(self.E, 1)), dtype=u8, device=dev)
        self._struct = _lib.ScacchiTree(
            B, Cn, self.A, S, self.E, *[t.data_ptr() for t in (
                self.parents_, self.children_, self.to_play_, self.node_outcome_, self.node_payload_,
                self.edge_outcome_, self.edge_payload_, self.value_prior_, self.value_alpha_,
                self.edge_alpha_, self.invalid_, self.embedding_)])

    # ---- C ABI --------------------------------------------------------------
    @property
    def struct(self) -> _lib.ScacchiTree:
        return self._struct

    def sref(self):
        return C.byref(self._struct)

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (
            self.parents_, self.children_, self.to_play_, self.node_outcome_, self.node_payload_,
            self.edge_outcome_, self.edge_payload_, self.value_prior_, self.value_alpha_, self.edge_alpha_,
            self.invalid_, self.embedding_))

    # ---- reference field names ----------------------------------------------
    @property
    def parents(self) -> torch.Tensor:
        return self.parents_

    @property
    def children_index(self) -> torch.Tensor:
        return self.children_[..., :self.A]

    @property
    def node_to_play(self) -> torch.Tensor:
        return self.to_play_

    @property
    def node_categorical_outcome(self) -> torch.Tensor:
        return self.node_outcome_

    @property
    def node_payload(self) -> torch.Tensor:
        return self.node_payload_

    @property
    def edge_categorical_outcome(self) -> torch.Tensor:
        return self.edge_outcome_[..., :self.A]

    @property
    def edge_payload(self) -> torch.Tensor:
        return self.edge_payload_[..., :self.A]

    @property
    def node_value_priors(self) -> torch.Tensor:
        return self.value_prior_

    @property
    def node_value_alpha(self) -> torch.Tensor:
        return self.value_alpha_

    @property
    def edge_alpha(self) -> torch.Tensor:
        return self.edge_alpha_[..., :self.A, :]

    @property
    def invalid_actions(self) -> torch.Tensor:
        return self.invalid_[..., :self.A].bool()

    @property
    def embeddings(self) -> Any:
        if self.codec is None:
            return None
        return self.codec.unpack(self.embedding_[..., :self.E])

    @property
    def num_actions(self) -> int:
        return self.A

    @property
    def num_simulations(self) -> int:
        return self.capacity - 1

    @property
    def searchable_actions(self) -> torch.Tensor:
        return ~self.invalid_actions & (self.edge_categorical_outcome == NO_OUTCOME)

    @property
    def root_action_alpha(self) -> torch.Tensor:
        return self.summary().alpha

    @property
    def root_stored_edge_alpha(self) -> torch.Tensor:
        return self.edge_alpha[:, self.ROOT_INDEX]

    @property
    def root_edge_payload(self) -> torch.Tensor:
        return self.edge_payload[:, self.ROOT_INDEX]

    @property
    def root_value_alpha(self) -> torch.Tensor:
        return self.node_value_alpha[:, self.ROOT_INDEX]

    @property
    def root_invalid_actions(self) -> torch.Tensor:
        return self.invalid_actions[:, self.ROOT_INDEX]

    def summary(self) -> SearchSummary:
        """tree.py:212-242, computed by the summary kernel."""
        B, A, dev = self.batch, self.A, self.device
        out = SearchSummary(
            torch.empty((B, A), dtype=torch.float32, device=dev),
            torch.empty((B, A, 2), dtype=torch.float32, device=dev),
            torch.empty((B, 2), dtype=torch.float32, device=dev),
            torch.empty((B, A), dtype=torch.int8, device=dev),
            torch.empty((B, A), dtype=torch.int32, device=dev),
            torch.empty((B,), dtype=torch.int8, device=dev),
            torch.empty((B,), dtype=torch.int32, device=dev))
        _lib.check(_lib.lib().scacchi_summary(
            self.sref(), *[ptr(getattr(out, f.name)) for f in dataclasses.fields(out)], stream_handle(dev)),
            "summary")
        return out


# --------------------------------------------------------------------------
# update views (tree.py:16-83)
# --------------------------------------------------------------------------

@dataclasses.dataclass(frozen=True)
class PosteriorUpdate:
    edge_alpha: torch.Tensor
    edge_payload: torch.Tensor
    value_alpha: torch.Tensor


@dataclasses.dataclass(frozen=True)
class NodeView:
    index: torch.Tensor
    embedding: Any
    value_prior: torch.Tensor
    value_alpha: torch.Tensor
    node_payload: torch.Tensor
    edge_alpha: torch.Tensor
    edge_payload: torch.Tensor
    edge_categorical_outcome: torch.Tensor
    to_play: torch.Tensor
    invalid_actions: torch.Tensor


@dataclasses.dataclass(frozen=True)
class ChildrenView:
    index: torch.Tensor
    visited: torch.Tensor
    embedding_table: Any
    value_prior: torch.Tensor
    value_alpha: torch.Tensor
    node_payload: torch.Tensor
    categorical_outcome: torch.Tensor
    to_play: torch.Tensor


@dataclasses.dataclass(frozen=True)
class LeafView:
    action: torch.Tensor
    value_alpha: torch.Tensor
    to_play: torch.Tensor
    active: torch.Tensor


@dataclasses.dataclass(frozen=True)
class PosteriorUpdateContext:
    node: NodeView
    children: ChildrenView
    leaf: LeafView
    active: torch.Tensor

    def replace(self, **kw) -> "PosteriorUpdateContext":
        return dataclasses.replace(self, **kw)


def _as(t, dtype, device) -> torch.Tensor:
    return torch.as_tensor(t).to(device=device, dtype=dtype).contiguous()


def instantiate_tree_from_root(root, num_simulations: int, root_invalid_actions: torch.Tensor) -> Tree:
    """tree.py:245-277: allocate and write every slot's defaults."""
    return _init_tree(root, num_simulations, root_invalid_actions, full=True)


def _init_tree(root, num_simulations: int, root_invalid_actions, full: bool) -> Tree:
    logits = root.prior_logits
    if logits.dim() != 2:
        raise ValueError("prior_logits must be [batch, action]")
    B, A = logits.shape
    dev = logits.device
    if root.action_values.shape != (B, A, 2) or root.value.shape != (B, 2):
        raise ValueError(
            "native search supports binary outcomes only: value [B, 2], action_values [B, A, 2]; "
            f"got {tuple(root.value.shape)} and {tuple(root.action_values.shape)}")
    if tuple(root_invalid_actions.shape) != (B, A):
        raise ValueError("root_invalid_actions must be [batch, action]")
    codec = EmbeddingCodec(root.embedding) if root.embedding is not None else None
    tree = Tree(B, num_simulations + 1, A, codec, dev)
    emb = codec.pack(root.embedding, B, dev) if codec is not None and codec.nbytes else None
    f32 = torch.float32
    args = (_as(root.value, f32, dev), _as(root.action_values, f32, dev),
            _as(root_invalid_actions, torch.uint8, dev), _as(root.terminal_outcome, torch.int8, dev),
            _as(root.to_play, torch.int32, dev))
    _lib.check(_lib.lib().scacchi_tree_init(tree.sref(), *[ptr(a) for a in args], ptr(emb), int(full),
                                            stream_handle(dev)), "tree_init")
    tree._keepalive = (args, emb)
    return tree
