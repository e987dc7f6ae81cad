"""tcgen05 residual tower (AZDirichletNet leaf evaluation) against fp32 torch.

* one padded-layout conv3x3 per epilogue mode against torch.conv2d in fp32 on
  the same 16-bit operands, with one product per K step and with split
  operands (hi + lo activations, and weights for three products);
* the whole network against the reference restated in torch
  (oracle/network_ref.py): tightly against the emulation of the kernel's own
  rounding points, and against pure fp32 on all 16384 boards of the tower
  workload: the default precision within 2e-2 max-abs on logits, log alpha_v
  and log alpha_q with >= 99.5 % policy-argmax agreement.
"""

import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROWS_PER_BOARD = 100


def padded_rows(boards: int) -> int:
    return (boards * ROWS_PER_BOARD + 127) // 128 * 128


def to_padded(act: np.ndarray, rows: int) -> np.ndarray:
    """[E, 9, 9, 128] -> padded-flat [rows, 128] (zero rows / columns)."""
    E = act.shape[0]
    out = np.zeros((rows, 128), np.float32)
    v = out[:E * ROWS_PER_BOARD].reshape(E, 10, 10, 128)
    v[:, 1:, :9, :] = act
    return out


def from_padded(buf: np.ndarray, boards: int) -> np.ndarray:
    return buf[:boards * ROWS_PER_BOARD].reshape(boards, 10, 10, -1)[:, 1:, :9, :]


def half(x: np.ndarray, fp16: bool) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.float16 if fp16 else torch.bfloat16)


def conv_ref(act: torch.Tensor, w_tap_out_in: torch.Tensor, bias: np.ndarray) -> torch.Tensor:
    """fp32 SAME conv of [E,9,9,C] with weights [9][out][in]."""
    w = w_tap_out_in.float().reshape(3, 3, 128, 128).permute(2, 3, 0, 1)  # out, in, ky, kx
    y = torch.nn.functional.conv2d(act.float().permute(0, 3, 1, 2), w, torch.from_numpy(bias), padding=1)
    return y.permute(0, 2, 3, 1)


@pytest.mark.parametrize("fp16", [False, True], ids=["bf16", "fp16"])
@pytest.mark.parametrize("mode", [0, 1, 2], ids=["conv1", "conv2", "heads"])
def test_single_conv_layer(cuda, mode, fp16):
    from scacchi_b200 import _lib

    rng = np.random.default_rng(10 + mode + 3 * fp16)
    E = 37  # 3700 rows: 29 tiles, the last one partial
    rows = padded_rows(E)
    act = np.maximum(rng.standard_normal((E, 9, 9, 128)), 0).astype(np.float32)
    res = rng.standard_normal((E, 9, 9, 128)).astype(np.float32)
    w = (rng.standard_normal((9, 128, 128)) * np.sqrt(2 / 1152)).astype(np.float32)
    b = rng.standard_normal(128).astype(np.float32) * 0.1
    sc = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    sh = (0.1 * rng.standard_normal(128)).astype(np.float32)
    hw = rng.standard_normal((6, 128)).astype(np.float32) * 0.1
    hb = rng.standard_normal(6).astype(np.float32) * 0.1
    act_h, res_h, w_h = half(act, fp16), half(res, fp16), half(w, fp16)
    dev = "cuda"
    inp = half(to_padded(act_h.float().numpy(), rows), fp16).to(dev)
    resid = half(to_padded(res_h.float().numpy(), rows), fp16).to(dev)
    wt = w_h.contiguous().to(dev)
    out0 = torch.full((rows, 128), 7.0, dtype=inp.dtype, device=dev)
    out1 = torch.full((rows, 128), 7.0, dtype=inp.dtype, device=dev)
    head = torch.zeros((rows, 8), dtype=torch.float32, device=dev)
    tb, tsc, tsh = (torch.from_numpy(v).to(dev) for v in (b, sc, sh))
    thw, thb = torch.from_numpy(hw).to(dev), torch.from_numpy(hb).to(dev)
    p = lambda t: C.c_void_p(t.data_ptr())
    rc = _lib.lib().scacchi_conv3x3(p(inp), p(wt), p(tb), mode, E, int(fp16), p(tsc), p(tsh), p(resid), p(thw),
                                    p(thb), p(out0), p(out1), p(head), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert _lib.tower_error() == 0
    y = conv_ref(act_h, w_h, b)
    dt = torch.float16 if fp16 else torch.bfloat16
    ulp = 2.0 ** (-10 if fp16 else -7)
    if mode == 0:
        want = torch.relu(y).to(dt).float().numpy()
        got = out0.float().cpu().numpy()
        np.testing.assert_allclose(from_padded(got, E), want, rtol=2 * ulp, atol=1e-3)
        pad = got[:E * ROWS_PER_BOARD].reshape(E, 10, 10, 128)
        assert not pad[:, 0].any() and not pad[:, :, 9].any()
        assert not got[E * ROWS_PER_BOARD:].any()
        return
    x_new = (y + res_h.float()).to(dt).float()
    a = torch.relu(x_new * torch.from_numpy(sc) + torch.from_numpy(sh)).to(dt).float()
    if mode == 1:
        np.testing.assert_allclose(from_padded(out0.float().cpu().numpy(), E), x_new.numpy(), rtol=2 * ulp, atol=2e-3)
        np.testing.assert_allclose(from_padded(out1.float().cpu().numpy(), E), a.numpy(), rtol=4 * ulp, atol=4e-3)
        return
    want = torch.relu(a @ torch.from_numpy(hw).T + torch.from_numpy(hb)).numpy()
    got = from_padded(head.cpu().numpy(), E)[..., :6]
    np.testing.assert_allclose(got, want, rtol=2e-2, atol=2e-2)


# the fp32 residual stream keeps each row's channels permuted within their
# 32-channel block: channel 32 q + 8 m + l (l < 8, m < 4) at 32 q + 4 l + m
_C = np.arange(128)
X32_SLOT = (_C & ~31) | ((_C & 7) << 2) | ((_C >> 3) & 3)


def x32_stored(x: np.ndarray) -> np.ndarray:
    out = np.empty_like(x)
    out[..., X32_SLOT] = x
    return out


def x32_natural(y: np.ndarray) -> np.ndarray:
    return y[..., X32_SLOT]


def _split16(x: np.ndarray, fp16: bool):
    """x -> (hi, lo) 16-bit tensors with hi = round(x), lo = round(x - hi)."""
    hi = half(x, fp16)
    lo = half(x - hi.float().numpy(), fp16)
    return hi, lo


@pytest.mark.parametrize("natural_in", [0, 1], ids=["x32_permuted", "x32_natural_in"])
@pytest.mark.parametrize("terms", [2, 3])
@pytest.mark.parametrize("fp16", [False, True], ids=["bf16", "fp16"])
@pytest.mark.parametrize("mode", [0, 1, 2], ids=["conv1", "conv2", "heads"])
def test_single_conv_layer_split(cuda, mode, fp16, terms, natural_in):
    """Split operands: the accumulator receives W_hi (A_hi + A_lo) (+ W_lo
    A_hi), the epilogue writes each 16-bit output as a hi / lo pair and keeps
    the residual stream in fp32, read in the permuted channel order (or, for
    the first block, the stem's natural order) and written permuted."""
    if mode == 0 and natural_in:
        pytest.skip("conv1 does not read the residual stream")
    from scacchi_b200 import _lib

    rng = np.random.default_rng(100 + mode + 3 * fp16 + 7 * terms)
    E = 37
    rows = padded_rows(E)
    act = np.maximum(rng.standard_normal((E, 9, 9, 128)), 0).astype(np.float32)
    res = rng.standard_normal((E, 9, 9, 128)).astype(np.float32)
    w = (rng.standard_normal((9, 128, 128)) * np.sqrt(2 / 1152)).astype(np.float32)
    b = rng.standard_normal(128).astype(np.float32) * 0.1
    sc = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    sh = (0.1 * rng.standard_normal(128)).astype(np.float32)
    hw = rng.standard_normal((6, 128)).astype(np.float32) * 0.1
    hb = rng.standard_normal(6).astype(np.float32) * 0.1
    a_hi, a_lo = _split16(act, fp16)
    w_hi, w_lo = _split16(w, fp16)
    dev = "cuda"
    dt = torch.float16 if fp16 else torch.bfloat16
    inp = half(to_padded(a_hi.float().numpy(), rows), fp16).to(dev)
    inp_lo = half(to_padded(a_lo.float().numpy(), rows), fp16).to(dev)
    wt = (torch.stack([w_hi, w_lo]) if terms == 3 else w_hi).contiguous().to(dev)
    x32_in = to_padded(res, rows)
    x32 = torch.from_numpy(x32_in if natural_in else x32_stored(x32_in)).to(dev)
    out_hi = torch.full((rows, 128), 7.0, dtype=dt, device=dev)
    out_lo = torch.full((rows, 128), 7.0, dtype=dt, device=dev)
    head = torch.zeros((rows, 8), dtype=torch.float32, device=dev)
    tb, tsc, tsh = (torch.from_numpy(v).to(dev) for v in (b, sc, sh))
    thw, thb = torch.from_numpy(hw).to(dev), torch.from_numpy(hb).to(dev)
    p = lambda t: C.c_void_p(t.data_ptr())
    rc = _lib.lib().scacchi_conv3x3_split(p(inp), p(inp_lo), p(wt), p(tb), mode, E, int(fp16), terms, p(tsc),
                                          p(tsh), p(x32), natural_in, p(thw), p(thb), p(out_hi), p(out_lo), p(head),
                                          C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert _lib.tower_error() == 0
    y = conv_ref(a_hi.float() + a_lo.float(), w_hi, b)
    if terms == 3:
        y = y + conv_ref(a_hi, w_lo, np.zeros(128, np.float32))
    y = y.numpy()
    got_pair = (out_hi.float() + out_lo.float()).cpu().numpy()
    if mode == 0:
        want = np.maximum(y, 0)
        np.testing.assert_allclose(from_padded(got_pair, E), want, rtol=1e-4, atol=1e-4)
        # hi is the 16-bit rounding of the pair's value
        hi = from_padded(out_hi.float().cpu().numpy(), E)
        assert (hi == torch.from_numpy(from_padded(got_pair, E).copy()).to(dt).float().numpy()).mean() > 0.999
        pad = got_pair[:E * ROWS_PER_BOARD].reshape(E, 10, 10, 128)
        assert not pad[:, 0].any() and not pad[:, :, 9].any()
        assert not got_pair[E * ROWS_PER_BOARD:].any()
        return
    x_new = y + res
    a = np.maximum(x_new * sc + sh, 0)
    if mode == 1:
        # the residual stream is updated in place (the heads layer leaves it)
        np.testing.assert_allclose(from_padded(x32_natural(x32.cpu().numpy()), E), x_new, rtol=1e-4, atol=1e-4)
        np.testing.assert_allclose(from_padded(got_pair, E), a, rtol=1e-4, atol=1e-4)
        return
    want = np.maximum(a @ hw.T + hb, 0)
    np.testing.assert_allclose(from_padded(head.cpu().numpy(), E)[..., :6], want, rtol=1e-4, atol=1e-4)


def _tower_outputs(params, obs, precision):
    from scacchi_b200.network import AZDirichletNet

    net = AZDirichletNet(params, precision=precision)
    logits, av, aq = net(torch.from_numpy(obs).cuda())
    torch.cuda.synchronize()
    return (logits.cpu().numpy(), net.last_log_alpha_v.cpu().numpy(), net.last_log_alpha_q.cpu().numpy(),
            av.cpu().numpy(), aq.cpu().numpy())


# kernel vs the emulation of its own rounding points (block gain 0.5: no
# amplification), max-abs bound per precision
EMULATION_TOL = {"bf16": 4e-2, "fp16": 6e-3, "fp16x2": 1e-3, "bf16x3": 1e-3, "fp16x3": 1e-4}


@pytest.mark.parametrize("precision", sorted(EMULATION_TOL))
def test_tower_matches_rounding_emulation(cuda, precision):
    """Kernel arithmetic against the emulation of its own rounding points.

    Summation order differs (tensor cores vs torch), so a value sitting on a
    16-bit rounding boundary can round the other way, and a He-normal stack
    amplifies such flips layer by layer.  With block gain 0.5 the network
    does not amplify and the comparison is tight; the deviations on the
    amplifying workload are covered by the fp32 test below."""
    from oracle import network_ref as R
    from scacchi_b200 import _lib
    from scacchi_b200.network import init_params

    params = init_params(0, random_batchnorm=True, block_gain=0.5)
    obs = R.observations(192, seed=1)
    got = _tower_outputs(params, obs, precision)
    want = R.forward(params, obs, precision=precision)
    assert _lib.tower_error() == 0
    tol = EMULATION_TOL[precision]
    for g, w, name in zip(got[:3], want, ("logits", "log_alpha_v", "log_alpha_q")):
        err = np.abs(g - w).max()
        assert err < tol, f"{name}: max abs {err}"
    np.testing.assert_allclose(got[3], np.exp(got[1]), rtol=1e-5)
    np.testing.assert_allclose(got[4], np.exp(got[2]), rtol=1e-5)


TOWER_BOARDS = 16384


@pytest.fixture(scope="module")
def tower_workload():
    """The tower workload (He-normal weights on every layer, seed 0, {0,1}
    planes of density 0.4, 16384 boards) and its fp32 outputs, computed by
    the restated network on the GPU with TF32 off."""
    from oracle import network_ref as R
    from scacchi_b200.network import init_params

    params = init_params(0)
    obs = R.observations(TOWER_BOARDS, seed=0)
    ref = R.forward(params, obs, device="cuda")
    torch.cuda.synchronize()
    return params, obs, ref


def _errors(got, ref):
    err = [float(np.abs(g - w).max()) for g, w in zip(got[:3], ref)]
    agree = float((got[0].argmax(1) == ref[0].argmax(1)).mean())
    return err, agree


def test_fp32_checker_on_gpu_matches_cpu(cuda, tower_workload):
    """The GPU run of the fp32 checker agrees with its CPU run (512 boards)."""
    from oracle import network_ref as R

    params, obs, ref = tower_workload
    cpu = R.forward(params, obs[:512])
    for c, g in zip(cpu, ref):
        np.testing.assert_allclose(g[:512], c, rtol=1e-4, atol=1e-4)


def test_default_precision_meets_the_stated_tolerance(cuda, tower_workload):
    """The default tower precision (bf16x3: bf16 operands split into hi + lo,
    three products, fp32 residual stream) on all 16384 boards of the tower
    workload: < 2e-2 max-abs on logits, log alpha_v and log alpha_q, and
    >= 99.5 % policy-argmax agreement with the fp32 network."""
    from scacchi_b200.network import DEFAULT_PRECISION

    params, obs, ref = tower_workload
    err, agree = _errors(_tower_outputs(params, obs, DEFAULT_PRECISION), ref)
    print(f"{DEFAULT_PRECISION}: max abs logits/lav/laq {err} argmax {agree}")
    assert err[0] < 2e-2 and err[1] < 2e-2 and err[2] < 2e-2
    assert agree >= 0.995


@pytest.mark.parametrize("seed, random_batchnorm", [(1, False), (5, True)])
def test_default_precision_holds_on_other_weights(cuda, seed, random_batchnorm):
    """The default precision within the stated tolerance on two more weight
    sets (16384 boards each; seed 5 with non-trivial BatchNorm statistics).
    fp16x2 is not the default because on these weights it leaves the bound:
    log alpha_q max-abs 0.036 (seed 1) and 0.045 (seed 5), against bf16x3's
    0.002 and 0.0015."""
    from oracle import network_ref as R
    from scacchi_b200.network import DEFAULT_PRECISION, init_params

    params = init_params(seed, random_batchnorm=random_batchnorm)
    obs = R.observations(TOWER_BOARDS, seed=seed)
    ref = R.forward(params, obs, device="cuda")
    err, agree = _errors(_tower_outputs(params, obs, DEFAULT_PRECISION), ref)
    print(f"seed {seed}: {DEFAULT_PRECISION} max abs logits/lav/laq {err} argmax {agree}")
    assert max(err) < 2e-2 and agree >= 0.995


@pytest.mark.parametrize("precision", ["bf16", "fp16", "fp16x2", "fp16x3"])
def test_other_precisions_against_fp32(cuda, tower_workload, precision):
    """The other precisions on the same 16384 boards, held to the deviation
    their 16-bit rounding implies (CPU emulation of each on this workload:
    bf16 0.14 / 0.25 / 0.25 with 97.6 % argmax agreement, the reference's own
    bf16 model 0.13 / 0.28 / 0.27 with 96.9 %; fp16 0.017 / 0.023 / 0.029,
    99.7 %; fp16x2 0.011 / 0.013 / 0.017; fp16x3 ~1e-4).  Only the split
    precisions reach the 2e-2 bound."""
    params, obs, ref = tower_workload
    err, agree = _errors(_tower_outputs(params, obs, precision), ref)
    print(f"{precision}: max abs logits/lav/laq {err} argmax {agree}")
    bound, min_agree = {"bf16": (0.4, 0.95), "fp16": (0.045, 0.99), "fp16x2": (2e-2, 0.995),
                        "fp16x3": (2e-3, 0.999)}[precision]
    assert max(err) < bound and agree >= min_agree


@pytest.mark.parametrize("boards", [1, 2, 37, 1281])
def test_ragged_board_counts_match_emulation(cuda, boards):
    """Board counts whose padded rows end inside a tile (the last tile's
    rows past the boards are padding) and tiny batches: the default
    precision against the emulation of its rounding points, and the same
    outputs when the boards are evaluated inside a larger batch."""
    from oracle import network_ref as R
    from scacchi_b200.network import DEFAULT_PRECISION, init_params

    params = init_params(3, random_batchnorm=True, block_gain=0.5)
    obs = R.observations(boards + 5, seed=boards)
    got = _tower_outputs(params, obs[:boards], DEFAULT_PRECISION)
    want = R.forward(params, obs[:boards], precision=DEFAULT_PRECISION)
    for g, w in zip(got[:3], want):
        assert np.abs(g - w).max() < EMULATION_TOL[DEFAULT_PRECISION]
    more = _tower_outputs(params, obs, DEFAULT_PRECISION)
    for g, m in zip(got, more):
        np.testing.assert_allclose(g, m[:boards], rtol=2e-6, atol=2e-6)


def test_forward_is_deterministic(cuda, tower_workload):
    """Two forwards of the same boards give the same bits (no atomics in
    the reductions)."""
    params, obs, _ = tower_workload
    a = _tower_outputs(params, obs[:2048], None)
    b = _tower_outputs(params, obs[:2048], None)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)
