"""AZDirichletNet leaf evaluator (network.py:338-524 of the reference) on B200.

Parameters use flax's layout (conv kernels HWIO, dense kernels [in, out],
BatchNorm scale/bias/mean/var), so a trained flax state converts one to one.
``fold`` turns them into the kernels' inference form: bf16 conv weights
[tap][out][in] with the BatchNorm after each block's first conv folded in,
per-channel scale/shift for the pre-activation BatchNorms, and the heads'
1x1 convolutions with their BatchNorm folded.  ``AZDirichletNet`` runs the
tcgen05 tower (csrc/tower.cu) and returns (logits, alpha_v, alpha_q) like the
reference module with ``train=False``.

Scope: resnet_v2, 9x9 boards, binary outcomes, direct log-concentration
heads (the Hex recipe: hex.yaml).
"""

from __future__ import annotations

import ctypes as C
import dataclasses
import math

import numpy as np
import torch

from . import _lib
from .dirichlet_mctx.tree import ptr, stream_handle

BN_EPS = 1e-5  # flax nnx.BatchNorm default epsilon
HEAD_CHANNELS = 6

# Tensor-core precision of the tower: name -> (fp16 operands, products per
# K step).  One product rounds activations and weights to 16 bits and keeps
# the residual stream in 16 bits, like the reference's bf16 model
# (compute_dtype bf16); two products add A_lo W for activations split as hi
# + lo; three add A_hi W_lo as well (weights split too).  Split operands
# keep the residual stream in fp32.  Measured on the He-normal tower
# workload (16384 boards) against the fp32 network: bf16 0.14 / 0.25 / 0.25
# max-abs on logits / log alpha_v / log alpha_q (97.6 % argmax agreement),
# the reference's own bf16 model 0.13 / 0.28 / 0.27 (96.9 %), fp16 0.017 /
# 0.023 / 0.029; bf16x3 stays near 3e-4.
PRECISIONS = {"bf16": (False, 1), "fp16": (True, 1), "fp16x2": (True, 2), "bf16x3": (False, 3),
              "fp16x3": (True, 3)}
DEFAULT_PRECISION = "bf16x3"


@dataclasses.dataclass
class BatchNormParams:
    scale: np.ndarray
    bias: np.ndarray
    mean: np.ndarray
    var: np.ndarray

    def affine(self) -> tuple[np.ndarray, np.ndarray]:
        """Inference form y = x * s + t (running statistics)."""
        s = self.scale / np.sqrt(self.var + BN_EPS)
        return s.astype(np.float32), (self.bias - self.mean * s).astype(np.float32)


@dataclasses.dataclass
class AZDirichletParams:
    """flax-layout parameters of AZDirichletNet (resnet_v2, binary outcomes)."""

    num_actions: int
    conv_w: np.ndarray                   # [3, 3, Cin, 128]
    conv_b: np.ndarray
    blocks: list                         # per block: dict bn1, conv1_w, conv1_b, bn2, conv2_w, conv2_b
    bn: BatchNormParams                  # final trunk BN
    policy_conv_w: np.ndarray            # [1, 1, 128, 2]
    policy_conv_b: np.ndarray
    policy_bn: BatchNormParams
    policy_w: np.ndarray                 # [162, A]
    policy_b: np.ndarray
    value_conv_w: np.ndarray             # [1, 1, 128, 1]
    value_conv_b: np.ndarray
    value_bn: BatchNormParams
    value_w: np.ndarray                  # [81, 128]
    value_b: np.ndarray
    value_dir_w: np.ndarray              # [128, 2]
    value_dir_b: np.ndarray
    value_conc_w: np.ndarray             # [128, 1]
    value_conc_b: np.ndarray
    q_dir_conv_w: np.ndarray             # [1, 1, 128, 2]
    q_dir_conv_b: np.ndarray
    q_dir_bn: BatchNormParams
    q_dir_w: np.ndarray                  # [162, 128]
    q_dir_b: np.ndarray
    q_dir_out_w: np.ndarray              # [128, 2A]
    q_dir_out_b: np.ndarray
    q_conc_conv_w: np.ndarray            # [1, 1, 128, 1]
    q_conc_conv_b: np.ndarray
    q_conc_bn: BatchNormParams
    q_conc_w: np.ndarray                 # [81, 128]
    q_conc_b: np.ndarray
    q_conc_out_w: np.ndarray             # [128, A]
    q_conc_out_b: np.ndarray


def init_params(seed: int = 0, *, num_actions: int = 82, in_planes: int = 4, channels: int = 128,
                num_blocks: int = 6, he_all_layers: bool = True, random_batchnorm: bool = False,
                initial_concentration: float = 3.1, block_gain: float = 1.0) -> AZDirichletParams:
    """He-normal weights (std sqrt(2 / fan_in)), zero biases.

    ``he_all_layers=False`` reproduces the reference's random init, whose
    output heads (policy_linear, value/Q mean and concentration outputs) are
    zero-initialised with the concentration biases at log(c0)
    (network.py:395-458): constant outputs.  ``random_batchnorm`` draws
    non-trivial BatchNorm statistics (for folding tests); otherwise BatchNorm
    is at its init (scale 1, bias 0, mean 0, var 1).  ``block_gain`` scales
    the residual blocks' conv weights (1: He-normal)."""
    rng = np.random.default_rng(seed)
    f32 = np.float32

    def he(shape, fan_in):
        return (rng.standard_normal(shape) * math.sqrt(2.0 / fan_in)).astype(f32)

    def zeros(*shape):
        return np.zeros(shape, f32)

    def bn(c):
        if random_batchnorm:
            return BatchNormParams(rng.uniform(0.6, 1.4, c).astype(f32), (0.1 * rng.standard_normal(c)).astype(f32),
                                   (0.1 * rng.standard_normal(c)).astype(f32), rng.uniform(0.6, 1.6, c).astype(f32))
        return BatchNormParams(np.ones(c, f32), zeros(c), zeros(c), np.ones(c, f32))

    def head(shape, fan_in, bias_value=0.0):
        if he_all_layers:
            return he(shape, fan_in), zeros(shape[-1])
        return zeros(*shape), np.full(shape[-1], bias_value, f32)

    A, Ch = num_actions, channels
    conc0 = math.log(initial_concentration)
    blocks = []
    for _ in range(num_blocks):
        blocks.append(dict(bn1=bn(Ch), conv1_w=block_gain * he((3, 3, Ch, Ch), 9 * Ch), conv1_b=zeros(Ch),
                           bn2=bn(Ch), conv2_w=block_gain * he((3, 3, Ch, Ch), 9 * Ch), conv2_b=zeros(Ch)))
    pw, pb = head((162, A), 162)
    vdw, vdb = head((Ch, 2), Ch)
    vcw, vcb = head((Ch, 1), Ch, conc0)
    qow, qob = head((Ch, 2 * A), Ch)
    qcw, qcb = head((Ch, A), Ch, conc0)
    return AZDirichletParams(
        num_actions=A, conv_w=he((3, 3, in_planes, Ch), 9 * in_planes), conv_b=zeros(Ch), blocks=blocks, bn=bn(Ch),
        policy_conv_w=he((1, 1, Ch, 2), Ch), policy_conv_b=zeros(2), policy_bn=bn(2), policy_w=pw, policy_b=pb,
        value_conv_w=he((1, 1, Ch, 1), Ch), value_conv_b=zeros(1), value_bn=bn(1), value_w=he((81, Ch), 81),
        value_b=zeros(Ch), value_dir_w=vdw, value_dir_b=vdb, value_conc_w=vcw, value_conc_b=vcb,
        q_dir_conv_w=he((1, 1, Ch, 2), Ch), q_dir_conv_b=zeros(2), q_dir_bn=bn(2), q_dir_w=he((162, Ch), 162),
        q_dir_b=zeros(Ch), q_dir_out_w=qow, q_dir_out_b=qob, q_conc_conv_w=he((1, 1, Ch, 1), Ch),
        q_conc_conv_b=zeros(1), q_conc_bn=bn(1), q_conc_w=he((81, Ch), 81), q_conc_b=zeros(Ch), q_conc_out_w=qcw,
        q_conc_out_b=qcb)


def _half_bits(x: np.ndarray, fp16: bool) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 / float16 bit patterns."""
    t = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.float16 if fp16 else torch.bfloat16)
    return t.view(torch.int16).numpy().view(np.uint16)


@dataclasses.dataclass
class FoldedWeights:
    """Inference-form weights on the device plus the C-ABI struct."""

    tensors: dict
    struct: _lib.TowerWeights
    num_actions: int
    in_planes: int


def fold(p: AZDirichletParams, device="cuda", fp16: bool = False, terms: int = 1) -> FoldedWeights:
    Ch = p.conv_w.shape[-1]
    nb = len(p.blocks)
    dev = torch.device(device)
    scales, shifts, conv_w, conv_b = [], [], [], []
    for blk in p.blocks:
        s1, t1 = blk["bn1"].affine()
        scales.append(s1)
        shifts.append(t1)
        s2, t2 = blk["bn2"].affine()
        w1 = blk["conv1_w"] * s2[None, None, None, :]            # fold BN2 into conv1
        b1 = blk["conv1_b"] * s2 + t2
        for w, b in ((w1, b1), (blk["conv2_w"], blk["conv2_b"])):
            # HWIO [3,3,in,out] -> [tap][out][in]
            conv_w.append(np.transpose(w.reshape(9, Ch, Ch), (0, 2, 1)))
            conv_b.append(b)
    s, t = p.bn.affine()
    scales.append(s)
    shifts.append(t)
    head_w, head_b = [], []
    for cw, cb, bnp in ((p.policy_conv_w, p.policy_conv_b, p.policy_bn), (p.value_conv_w, p.value_conv_b, p.value_bn),
                        (p.q_dir_conv_w, p.q_dir_conv_b, p.q_dir_bn), (p.q_conc_conv_w, p.q_conc_conv_b, p.q_conc_bn)):
        hs, ht = bnp.affine()
        w = cw.reshape(Ch, -1) * hs[None, :]
        head_w.append(w.T)
        head_b.append(cb * hs + ht)
    A = p.num_actions
    host = dict(
        stem_w=p.conv_w.reshape(9, -1, Ch).astype(np.float32), stem_b=p.conv_b, bn_scale=np.stack(scales),
        bn_shift=np.stack(shifts), conv_b=np.stack(conv_b), head_w=np.concatenate(head_w, 0),
        head_b=np.concatenate(head_b, 0), policy_w=p.policy_w, policy_b=p.policy_b, value_w1=p.value_w,
        value_b1=p.value_b, value_mean_w=p.value_dir_w, value_mean_b=p.value_dir_b,
        value_conc_w=p.value_conc_w.reshape(-1), value_conc_b=p.value_conc_b, qdir_w1=p.q_dir_w, qdir_b1=p.q_dir_b,
        qdir_w2=p.q_dir_out_w, qdir_b2=p.q_dir_out_b, qconc_w1=p.q_conc_w, qconc_b1=p.q_conc_b,
        qconc_w2=p.q_conc_out_w, qconc_b2=p.q_conc_out_b)
    tensors = {k: torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(dev) for k, v in host.items()}
    w = np.stack(conv_w)                                           # [layers, 9, out, in]
    hi = _half_bits(w, fp16)
    if terms == 3:
        # [layers][hi, lo]: lo = the remainder w - hi rounded to 16 bits
        hi_f = torch.from_numpy(hi.view(np.int16)).view(torch.float16 if fp16 else torch.bfloat16).float().numpy()
        hi = np.stack([hi, _half_bits(w - hi_f, fp16)], axis=1)
    tensors["conv_w"] = torch.from_numpy(np.ascontiguousarray(hi).view(np.int16)).to(dev)
    in_planes = p.conv_w.shape[2]
    st = _lib.TowerWeights(nb, Ch, 9, 9, in_planes, A, int(fp16), int(terms),
                           *[tensors[k].data_ptr() for k in _lib.TowerWeights.POINTERS])
    return FoldedWeights(tensors, st, A, in_planes)


class AZDirichletNet:
    """Callable leaf evaluator: obs [B, 9, 9, planes] -> (logits [B, A],
    alpha_v [B, 2], alpha_q [B, A, 2]); ``log_alphas`` gives the logs."""

    def __init__(self, params: AZDirichletParams, device="cuda", fp16: bool | None = None,
                 precision: str | None = None):
        """``precision``: a name of PRECISIONS (default DEFAULT_PRECISION,
        the split bf16 operands whose outputs stay within 2e-2 of the fp32
        network).  ``fp16=False`` / ``True`` alone selects the one-product
        "bf16" (the reference's compute dtype) / "fp16" tower."""
        if precision is None:
            precision = DEFAULT_PRECISION if fp16 is None else ("fp16" if fp16 else "bf16")
        if precision not in PRECISIONS:
            raise ValueError(f"unknown tower precision {precision!r}; expected one of {sorted(PRECISIONS)}")
        self.params = params
        self.device = torch.device(device)
        self.precision = precision
        self.fp16, self.terms = PRECISIONS[precision]
        self.weights = fold(params, self.device, self.fp16, self.terms)
        self._ws = None
        self.last_log_alpha_v = None
        self.last_log_alpha_q = None

    @property
    def num_actions(self) -> int:
        return self.weights.num_actions

    def __call__(self, obs: torch.Tensor, train: bool = False):
        if train:
            raise ValueError("this backend implements inference (train=False) only")
        B = obs.shape[0]
        A, dev = self.num_actions, self.device
        x = obs.to(device=dev, dtype=torch.float32).contiguous()
        if tuple(x.shape[1:]) != (9, 9, self.weights.in_planes):
            raise ValueError(f"observation must be [B, 9, 9, {self.weights.in_planes}], got {tuple(obs.shape)}")
        need = int(_lib.lib().scacchi_tower_workspace_bytes(B))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty((need,), dtype=torch.uint8, device=dev)
        logits = torch.empty((B, A), dtype=torch.float32, device=dev)
        lav = torch.empty((B, 2), dtype=torch.float32, device=dev)
        laq = torch.empty((B, A, 2), dtype=torch.float32, device=dev)
        av = torch.empty((B, 2), dtype=torch.float32, device=dev)
        aq = torch.empty((B, A, 2), dtype=torch.float32, device=dev)
        _lib.check(_lib.lib().scacchi_tower_forward(C.byref(self.weights.struct), ptr(x), B, ptr(self._ws),
                                                    ptr(logits), ptr(lav), ptr(laq), ptr(av), ptr(aq),
                                                    stream_handle(dev)), "tower_forward")
        self.last_log_alpha_v, self.last_log_alpha_q = lav, laq
        return logits, av, aq
