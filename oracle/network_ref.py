"""fp32 reference of AZDirichletNet.__call__(x, train=False) in torch (CPU).

TEST INFRASTRUCTURE ONLY: the checker for the tcgen05 tower.  It follows
the reference's module structure (network.py:239-254, 460-524: NHWC,
SAME-padded 3x3 convolutions with bias, BatchNorm with running statistics,
ReLU, flatten in (y, x, channel) order, dirichlet_from_logits with direct
log-concentration heads clipped to [-80, 80]).

``precision`` (a name of scacchi_b200.network.PRECISIONS) instead rounds at
the kernel's rounding points (folded 16-bit weights, 16-bit activations
between layers, fp32 accumulation; split operands as hi + lo pairs with an
fp32 residual stream), which isolates the kernel's arithmetic from its
16-bit quantisation.  ``emulate_bf16=True`` is precision "bf16" ("fp16"
with ``fp16``).
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from scacchi_b200.network import BN_EPS, PRECISIONS, AZDirichletParams, BatchNormParams


_DEV = ["cpu"]  # where forward() runs its torch ops (set per call)


def _t(x) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        return x.to(device=_DEV[0], dtype=torch.float32)
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(_DEV[0])


def _conv(x_nhwc: torch.Tensor, w_hwio, b) -> torch.Tensor:
    w = _t(w_hwio).permute(3, 2, 0, 1)  # OIHW
    k = w.shape[-1]
    y = F.conv2d(x_nhwc.permute(0, 3, 1, 2), w, _t(b), padding=k // 2)
    return y.permute(0, 2, 3, 1)


def _bn(x: torch.Tensor, p: BatchNormParams) -> torch.Tensor:
    return (x - _t(p.mean)) / torch.sqrt(_t(p.var) + BN_EPS) * _t(p.scale) + _t(p.bias)


def _bf16(x: torch.Tensor) -> torch.Tensor:
    return x.to(_HALF[0]).to(torch.float32)


_HALF = [torch.bfloat16]


def _dirichlet(mean_logits: torch.Tensor, conc_logit: torch.Tensor):
    c = torch.clamp(conc_logit, -80.0, 80.0)
    log_alpha = c[..., None] + torch.log_softmax(mean_logits, dim=-1)
    return log_alpha


def _split_conv(a: torch.Tensor, w_hwio: np.ndarray, b, terms: int) -> torch.Tensor:
    """conv of split operands: W_hi (A_hi + A_lo) [+ W_lo A_hi] (terms 2 [3])."""
    a_hi = _bf16(a)
    a_lo = _bf16(a - a_hi)
    w = _t(w_hwio)
    w_hi = _bf16(w)
    y = _conv(a_hi + a_lo, w_hi, b)
    if terms == 3:
        y = y + _conv(a_hi, _bf16(w - w_hi), np.zeros_like(b))
    return y


def forward(p: AZDirichletParams, obs: np.ndarray, emulate_bf16: bool = False, fp16: bool = False,
            precision: str | None = None, device: str = "cpu"):
    """obs [B, 9, 9, planes] -> (logits [B, A], log_alpha_v [B, 2],
    log_alpha_q [B, A, 2]) as float32 numpy arrays, in fp32, or emulating
    the kernel at ``precision``.  ``device="cuda"`` runs the same torch ops
    on the GPU in true fp32 (TF32 off for convolutions and matmuls)."""
    _DEV[0] = device
    if device != "cpu":
        torch.backends.cudnn.allow_tf32 = False
        torch.backends.cuda.matmul.allow_tf32 = False
    if precision is None and emulate_bf16:
        precision = "fp16" if fp16 else "bf16"
    terms = 1
    if precision is not None:
        fp16, terms = PRECISIONS[precision]
    _HALF[0] = torch.float16 if fp16 else torch.bfloat16
    with torch.no_grad():
        x = _t(obs)
        B = x.shape[0]
        A = p.num_actions
        if precision is not None and terms > 1:
            # split operands: fp32 residual stream and activations, each
            # convolution's input split into hi + lo at the conv
            s0, t0 = (_t(v) for v in p.blocks[0]["bn1"].affine())
            x = _conv(x, p.conv_w, p.conv_b)
            a = torch.relu(x * s0 + t0)
            nb = len(p.blocks)
            for i, blk in enumerate(p.blocks):
                s2, t2 = blk["bn2"].affine()
                h = torch.relu(_split_conv(a, blk["conv1_w"] * s2[None, None, None, :], blk["conv1_b"] * s2 + t2,
                                           terms))
                x = _split_conv(h, blk["conv2_w"], blk["conv2_b"], terms) + x
                nxt = p.blocks[i + 1]["bn1"] if i + 1 < nb else p.bn
                s, t = (_t(v) for v in nxt.affine())
                a = torch.relu(x * s + t)
            heads = []
            for cw, cb, bnp in ((p.policy_conv_w, p.policy_conv_b, p.policy_bn),
                                (p.value_conv_w, p.value_conv_b, p.value_bn),
                                (p.q_dir_conv_w, p.q_dir_conv_b, p.q_dir_bn),
                                (p.q_conc_conv_w, p.q_conc_conv_b, p.q_conc_bn)):
                hs, ht = bnp.affine()
                heads.append(torch.relu(_conv(a, cw * hs, cb * hs + ht)))
        elif precision is None:
            x = _conv(x, p.conv_w, p.conv_b)
            for blk in p.blocks:
                r = x
                y = torch.relu(_bn(x, blk["bn1"]))
                y = _conv(y, blk["conv1_w"], blk["conv1_b"])
                y = torch.relu(_bn(y, blk["bn2"]))
                y = _conv(y, blk["conv2_w"], blk["conv2_b"])
                x = y + r
            feat = torch.relu(_bn(x, p.bn))
            heads = []
            for cw, cb, bnp in ((p.policy_conv_w, p.policy_conv_b, p.policy_bn),
                                (p.value_conv_w, p.value_conv_b, p.value_bn),
                                (p.q_dir_conv_w, p.q_dir_conv_b, p.q_dir_bn),
                                (p.q_conc_conv_w, p.q_conc_conv_b, p.q_conc_bn)):
                heads.append(torch.relu(_bn(_conv(feat, cw, cb), bnp)))
        else:
            # the kernel's one-product arithmetic: BN folded, 16-bit weights and activations
            s0, t0 = (_t(v) for v in p.blocks[0]["bn1"].affine())
            x = _bf16(_conv(x, p.conv_w, p.conv_b))
            a = _bf16(torch.relu(x * s0 + t0))
            nb = len(p.blocks)
            for i, blk in enumerate(p.blocks):
                s2, t2 = blk["bn2"].affine()
                w1 = _bf16(_t(blk["conv1_w"] * s2[None, None, None, :]))
                b1 = blk["conv1_b"] * s2 + t2
                h = _bf16(torch.relu(_conv(a, w1, b1)))
                w2 = _bf16(_t(blk["conv2_w"]))
                x = _bf16(_conv(h, w2, blk["conv2_b"]) + x)
                nxt = p.blocks[i + 1]["bn1"] if i + 1 < nb else p.bn
                s, t = (_t(v) for v in nxt.affine())
                a = _bf16(torch.relu(x * s + t))
            heads = []
            for cw, cb, bnp in ((p.policy_conv_w, p.policy_conv_b, p.policy_bn),
                                (p.value_conv_w, p.value_conv_b, p.value_bn),
                                (p.q_dir_conv_w, p.q_dir_conv_b, p.q_dir_bn),
                                (p.q_conc_conv_w, p.q_conc_conv_b, p.q_conc_bn)):
                hs, ht = bnp.affine()
                heads.append(torch.relu(_conv(a, cw * hs, cb * hs + ht)))
        pol, val, qd, qc = heads
        logits = pol.reshape(B, -1) @ _t(p.policy_w) + _t(p.policy_b)
        v = torch.relu(val.reshape(B, -1) @ _t(p.value_w) + _t(p.value_b))
        lav = _dirichlet(v @ _t(p.value_dir_w) + _t(p.value_dir_b),
                         (v @ _t(p.value_conc_w) + _t(p.value_conc_b)).reshape(B))
        q = torch.relu(qd.reshape(B, -1) @ _t(p.q_dir_w) + _t(p.q_dir_b))
        qm = (q @ _t(p.q_dir_out_w) + _t(p.q_dir_out_b)).reshape(B, A, 2)
        c = torch.relu(qc.reshape(B, -1) @ _t(p.q_conc_w) + _t(p.q_conc_b))
        laq = _dirichlet(qm, c @ _t(p.q_conc_out_w) + _t(p.q_conc_out_b))
        return logits.cpu().numpy(), lav.cpu().numpy(), laq.cpu().numpy()


def observations(boards: int, seed: int = 0, density: float = 0.4, planes: int = 4) -> np.ndarray:
    """{0,1} observation planes with the given density (the tower workload)."""
    rng = np.random.default_rng(seed)
    return (rng.uniform(size=(boards, 9, 9, planes)) < density).astype(np.float32)
