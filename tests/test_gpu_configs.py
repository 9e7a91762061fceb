"""Parity of the CUDA path with the CPU oracle at the BASELINE configurations' full sizes.

* config 3 (bulk fcc Cu 10x10x10, 4,000 atoms, 120,000 edges, C=128, 4 layers): energy and
  forces of the default path (fused f16x3 blocks) against the fp64 oracle, and the f16x3
  range flag clear;
* config 4 (water box, 3,333 H2O, ~10,000 atoms, ~300,000 edges): energy, forces and stress
  against the oracle in fp32 (an fp64 oracle of this size needs tens of GB of host memory);
* config 2 (one message-passing layer at N = 20,000, E = 600,000): the fused message block and
  every per-op entry point, forward and backward, run at full size on the GPU and are checked on
  a fixed sample of 512 atoms and 4,096 edges. The oracle evaluates exactly the edges a sampled
  row depends on (a destination atom's incoming CSR segment; for node gradients every edge that
  touches the atom), in fp64, so no full-size fp64 tensor is built.

Bars (``north_star``): energy 1e-5 relative, forces 1e-4 eV/A max-abs; per-op tensors 2e-5
relative to the tensor's max magnitude (5e-5 for reductions over channels), as the small-size
op tests use."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.fixture(autouse=True)
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


def _rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp(min=1.0)).item()


def _as(data, dtype):
    return type(data)(**{**data.__dict__, "pos": data.pos.to(dtype), "cell": data.cell.to(dtype),
                         "cell_offsets": data.cell_offsets.to(dtype)})


def _e2e(system, stress: bool, oracle_dtype):
    """(CUDA result, oracle result) of one energy + forces (+ stress) evaluation."""
    import os

    from flash_uma_b200.linear import check_errors
    from flash_uma_b200.predict import Predictor
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
    from flash_uma_b200.systems import to_graph
    from flash_uma_b200.wrapper import ZeroAllocBackbone
    from oracle.model import OracleBackbone
    torch.set_num_threads(os.cpu_count() or 1)
    data = to_graph([system])
    off = SyntheticESCNMDBackbone(seed=0, stress=stress)
    head = make_energy_head(128, 128, seed=1)
    bb = ZeroAllocBackbone(copy.deepcopy(off).to(DEV))
    assert bb.ce.fused, "the default path at C = 128 is the fused f16x3 one"
    res = Predictor(bb, copy.deepcopy(head).to(DEV))(data.to(DEV), stress=stress)
    torch.cuda.synchronize()
    check_errors()    # no f16x3 range error (code 16) and no pipeline timeout at this size
    res = {k: v.cpu() for k, v in res.items()}
    if oracle_dtype == torch.float64:
        off, head = off.double(), head.double()
    # layer checkpointing bounds the oracle's host memory (config 3 in fp64: ~21 GB instead of ~54 GB)
    ref = Predictor(OracleBackbone(off, oracle_dtype, checkpoint_layers=True), head)(_as(data, oracle_dtype),
                                                                                  stress=stress)
    return res, ref


def _check_e2e(res, ref, stress):
    e, er = res["energy"].double(), ref["energy"].double()
    erel = ((e - er).abs() / er.abs().clamp(min=1.0)).max().item()
    ferr = (res["forces"].double() - ref["forces"].double()).abs().max().item()
    assert erel < 1e-5, erel
    assert ferr < 1e-4, ferr
    if stress:
        s, sr = res["stress"].double(), ref["stress"].double()
        assert (s - sr).abs().max().item() < 1e-4 * max(1.0, sr.abs().max().item())


def test_config3_matches_oracle():
    """BASELINE config 3 (the bench workload) end to end against the fp64 oracle."""
    from flash_uma_b200.systems import config3_system
    system = config3_system()
    res, ref = _e2e(system, stress=False, oracle_dtype=torch.float64)
    assert res["forces"].shape == (4000, 3)
    _check_e2e(res, ref, stress=False)


def test_config4_water_matches_oracle():
    """BASELINE config 4 (water box, energy + forces + stress) against the fp32 oracle."""
    from flash_uma_b200.systems import config4_system
    res, ref = _e2e(config4_system(), stress=True, oracle_dtype=torch.float32)
    assert res["forces"].shape[0] == 9999
    _check_e2e(res, ref, stress=True)


# ---------------------------------------------------------------------------------- config 2

N2, E2, C2, B2 = 20000, 600000, 128, 64


@pytest.fixture(scope="module")
def cfg2():
    """Full-size config-2 inputs on the device and the fixed sample (512 atoms, 4,096 edges)."""
    from flash_uma_b200 import ops
    from flash_uma_b200.systems import microbench_layer_inputs
    inp = microbench_layer_inputs(N=N2, E=E2, C=C2, seed=0)
    g = torch.Generator().manual_seed(123)
    atoms = torch.randperm(N2, generator=g)[:512].sort()[0]
    edges = torch.randperm(E2, generator=g)[:4096].sort()[0]
    d = {k: (v.to(DEV) if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}
    d["graph"] = ops.build_graph_csr(d["idx_i"], d["idx_j"], N2)
    d["Z"] = torch.full((N2,), 29, dtype=torch.long, device=DEV)
    d["batch"] = torch.zeros(N2, dtype=torch.long, device=DEV)
    d["offset"] = torch.linspace(0, 6.0, B2, device=DEV)
    d["coeff"] = float(-0.5 / (2.0 * (6.0 / (B2 - 1))) ** 2)
    d["csd"] = torch.randn(1, C2, generator=g).to(DEV)
    d["W_src"] = (torch.randn(100, C2, generator=g) * 0.5).to(DEV)
    d["W_tgt"] = (torch.randn(100, C2, generator=g) * 0.5).to(DEV)
    d["atoms"], d["edges"] = atoms, edges
    cpu = {k: inp[k] for k in ("idx_i", "idx_j", "shifts", "x")}
    in_s = torch.isin(cpu["idx_j"], atoms)
    touch = in_s | torch.isin(cpu["idx_i"], atoms)
    d["dst_in_s"] = in_s.nonzero().squeeze(1)         # edges whose destination is sampled
    d["touch_s"] = touch.nonzero().squeeze(1)         # edges with a sampled endpoint
    d["cpu"] = cpu
    return d


def _oracle_geometry(d, e):
    from oracle import ops as oops
    c = d["cpu"]
    N = N2
    return oops.precompute_geometry(torch.zeros(N, 3, dtype=torch.float64), torch.full((N,), 29), c["idx_i"][e],
                                    c["idx_j"][e], c["shifts"][e].double(), d["W_src"].cpu().double(),
                                    d["W_tgt"].cpu().double(), d["offset"].cpu().double(), d["coeff"], 6.0)


def test_config2_ops_full_size(cfg2):
    """Each per-op entry point forward + backward at N = 20,000, E = 600,000 on the GPU, checked on
    the sample: geometry (edges), LN-SiLU (rows), gather (edges; node gradient on atoms),
    gating (edges), rotate-scatter (atoms; edge gradients)."""
    from flash_uma_b200 import ops
    from oracle import ops as oops
    d = cfg2
    c = d["cpu"]
    S, Es = d["atoms"], d["edges"]
    g = torch.Generator().manual_seed(7)

    # geometry: forward rows and the per-edge shift gradient
    sh = d["shifts"].clone().requires_grad_(True)
    xe, wig, env = ops.precompute_geometry(d["pos"], d["Z"], d["idx_i"], d["idx_j"], sh, d["W_src"], d["W_tgt"],
                                           d["offset"], d["coeff"], 6.0, graph=d["graph"])
    g_xe = torch.randn(E2, B2 + 2 * C2, generator=g)
    g_wig, g_env = torch.randn(E2, 34, generator=g), torch.randn(E2, generator=g)
    (gs,) = torch.autograd.grad([xe, wig, env], [sh], [g_xe.to(DEV), g_wig.to(DEV), g_env.to(DEV)])
    sh_o = c["shifts"][Es].double().requires_grad_(True)
    from oracle import ops as _o
    xo, wo, eo = _o.precompute_geometry(torch.zeros(N2, 3, dtype=torch.float64), torch.full((N2,), 29),
                                        c["idx_i"][Es], c["idx_j"][Es], sh_o, d["W_src"].cpu().double(),
                                        d["W_tgt"].cpu().double(), d["offset"].cpu().double(), d["coeff"], 6.0)
    (gso,) = torch.autograd.grad([xo, wo, eo], [sh_o], [g_xe[Es].double(), g_wig[Es].double(), g_env[Es].double()])
    assert _rel(xe[Es.to(DEV)], xo) < 2e-5 and _rel(wig[Es.to(DEV)], wo) < 2e-5
    assert (env[Es.to(DEV)].cpu().double() - eo).abs().max().item() < 1e-5
    assert _rel(gs[Es.to(DEV)], gso) < 5e-5
    wig, env = wig.detach(), env.detach()
    del xe, gs, g_xe

    # LN-SiLU on [E, 128] rows
    x = torch.randn(E2, 128, generator=g) * 2 + 0.3
    gm, bt = 1 + 0.1 * torch.randn(128, generator=g), 0.1 * torch.randn(128, generator=g)
    xd = x.to(DEV).requires_grad_(True)
    y = ops.layer_norm_silu(xd, gm.to(DEV), bt.to(DEV))
    go = torch.randn(E2, 128, generator=g)
    (gx,) = torch.autograd.grad(y, [xd], go.to(DEV))
    xo = x[Es].double().requires_grad_(True)
    yo = oops.layer_norm_silu(xo, gm.double(), bt.double())
    (gxo,) = torch.autograd.grad(yo, [xo], go[Es].double())
    assert _rel(y[Es.to(DEV)], yo) < 2e-5 and _rel(gx[Es.to(DEV)], gxo) < 5e-5
    del x, xd, y, go, gx

    # gather: X rows of the sampled edges; g_rad / g_wigner rows; g_x on sampled atoms
    x = d["x"].clone().requires_grad_(True)
    rad = (torch.randn(E2, 12 * C2, generator=g)).to(DEV).requires_grad_(True)
    wg = wig.clone().requires_grad_(True)
    X = ops.gather_wigner_split(x, d["idx_i"], d["idx_j"], wg, rad, d["csd"], d["batch"], graph=d["graph"])
    gX = [torch.randn(E2, w * C2, generator=g) for w in (6, 8, 4)]
    gx, gw, gr = torch.autograd.grad(list(X), [x, wg, rad], [t.to(DEV) for t in gX])
    T = d["touch_s"]
    xo = c["x"].double().requires_grad_(True)
    wo = wig[T.to(DEV)].cpu().double().requires_grad_(True)
    ro = rad.detach()[T.to(DEV)].cpu().double().requires_grad_(True)
    Xo = oops.gather_wigner_split(xo, c["idx_i"][T], c["idx_j"][T], wo, ro, d["csd"].cpu().double(),
                                  torch.zeros(N2, dtype=torch.long))
    gxo, gwo, gro = torch.autograd.grad(list(Xo), [xo, wo, ro], [t[T].double() for t in gX])
    pos_in_T = torch.searchsorted(T, Es[torch.isin(Es, T)])
    Ese = Es[torch.isin(Es, T)]
    for a, b in zip(X, Xo):
        assert _rel(a[Ese.to(DEV)], b[pos_in_T]) < 2e-5
    assert _rel(gx[S.to(DEV)], gxo[S]) < 5e-5
    assert _rel(gw[Ese.to(DEV)], gwo[pos_in_T]) < 5e-5 and _rel(gr[Ese.to(DEV)], gro[pos_in_T]) < 2e-5
    del X, gX, gx, gw, gr, x, rad, wg

    # gating on the sampled edges
    Y = [torch.randn(E2, w * C2, generator=g) for w in (5, 4, 2)]
    Yd = [t.to(DEV).requires_grad_(True) for t in Y]
    Zc = ops.fused_gating_split(*Yd, C2)
    gZ = [torch.randn(E2, w * C2, generator=g) for w in (3, 4, 2)]
    gY = torch.autograd.grad(list(Zc), Yd, [t.to(DEV) for t in gZ])
    Yo = [t[Es].double().requires_grad_(True) for t in Y]
    Zo = oops.fused_gating_split(*Yo, C2)
    gYo = torch.autograd.grad(list(Zo), Yo, [t[Es].double() for t in gZ])
    for a, b in zip(Zc, Zo):
        assert _rel(a[Es.to(DEV)], b) < 2e-5
    for a, b in zip(gY, gYo):
        assert _rel(a[Es.to(DEV)], b) < 2e-5
    del Y, Yd, Zc, gZ, gY

    # rotate-scatter: sampled atoms' rows (their whole CSR segments), per-edge gradients
    Zs = [torch.randn(E2, w * C2, generator=g) for w in (3, 4, 2)]
    Zd = [t.to(DEV).requires_grad_(True) for t in Zs]
    wg = wig.clone().requires_grad_(True)
    en = env.clone().requires_grad_(True)
    xr = d["x"]
    out = ops.rotate_scatter_split(*Zd, wg, en, xr, d["idx_j"], d["graph"].dst_row_ptr, d["graph"].dst_col, N2)
    gout = torch.randn(N2, 9, C2, generator=g)
    gz0, gz1, gz2, gw, ge = torch.autograd.grad(out, Zd + [wg, en], gout.to(DEV))
    Dd = d["dst_in_s"]
    Zo = [t[Dd].double() for t in Zs]
    oo = oops.rotate_scatter_split(*Zo, wig[Dd.to(DEV)].cpu().double(), env[Dd.to(DEV)].cpu().double(),
                                   c["x"].double(), c["idx_j"][Dd], None, None, N2)
    assert _rel(out[S.to(DEV)], oo[S]) < 2e-5
    Zo = [t[Es].double().requires_grad_(True) for t in Zs]
    wo = wig[Es.to(DEV)].cpu().double().requires_grad_(True)
    eo = env[Es.to(DEV)].cpu().double().requires_grad_(True)
    oo = oops.rotate_scatter_split(*Zo, wo, eo, c["x"].double(), c["idx_j"][Es], None, None, N2)
    go = torch.autograd.grad(oo, Zo + [wo, eo], gout.double())
    for a, b in zip((gz0, gz1, gz2), go[:3]):
        assert _rel(a[Es.to(DEV)], b) < 2e-5
    assert _rel(gw[Es.to(DEV)], go[3]) < 5e-5 and _rel(ge[Es.to(DEV)], go[4]) < 5e-5


def test_config2_message_block_full_size(cfg2):
    """The production path of one layer (fused f16x3 message block: radial MLP, gather, conv1,
    gating, conv2, rotate-scatter) forward + backward at full size; x_mid and the node gradient
    on the sampled atoms, the Wigner / envelope / Gaussian-feature gradients on the sampled edges,
    against the fp64 oracle on the edges those rows depend on."""
    import torch.nn.functional as F

    from flash_uma_b200 import fused
    from flash_uma_b200.linear import FrozenLinear, check_errors
    from flash_uma_b200.model import PackedLayer
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone
    from oracle import ops as oops
    from oracle.model import OracleLayer
    d = cfg2
    c = d["cpu"]
    S, Es = d["atoms"], d["edges"]
    off = SyntheticESCNMDBackbone(num_layers=1, seed=0)
    layer = PackedLayer(copy.deepcopy(off.blocks[0]).to(DEV), C2, "f16x3").to(DEV)
    layer.rad.n_gauss = B2
    for lin in layer.modules():
        if isinstance(lin, FrozenLinear):
            lin.prepare()
    xe, wig, env = fused.geometry(d["pos"], d["Z"], d["idx_i"], d["idx_j"], d["shifts"], d["W_src"], d["W_tgt"],
                                  d["offset"], d["coeff"], 6.0, d["graph"])
    xe_p, x_gauss = xe
    g = torch.Generator().manual_seed(9)
    x_norm = (d["x"] * 0.7).clone().requires_grad_(True)
    x_in = d["x"].clone().requires_grad_(True)
    xg = x_gauss.detach().clone().requires_grad_(True)
    wg = wig.detach().clone().requires_grad_(True)
    en = env.detach().clone().requires_grad_(True)
    out = fused.message_block(layer, x_norm, x_in, (xe_p, xg), wg, en, d["csd"], d["idx_i"], d["idx_j"], d["batch"],
                              d["graph"])
    gmid = torch.randn(N2, 9, C2, generator=g)
    gxn, gxi, gg, gw, ge = torch.autograd.grad(out, [x_norm, x_in, xg, wg, en], gmid.to(DEV))
    torch.cuda.synchronize()
    check_errors()

    ol = OracleLayer(off.blocks[0].double(), C2, torch.float64)

    def edge_msgs(e, xn, xe_rows, w, v):
        rad = ol.rad(xe_rows)
        X0, X1, X2 = oops.gather_wigner_split(xn, c["idx_i"][e], c["idx_j"][e], w, rad, d["csd"].cpu().double(),
                                              torch.zeros(N2, dtype=torch.long))
        Y0, Y1, Y2 = F.linear(X0, ol.W1_m0, ol.b1_m0), F.linear(X1, ol.W1_m1), F.linear(X2, ol.W1_m2)
        Z0, Z1, Z2 = oops.fused_gating_split(Y0, Y1, Y2, C2)
        O0, O1, O2 = F.linear(Z0, ol.W2_m0, ol.b2_m0), F.linear(Z1, ol.W2_m1), F.linear(Z2, ol.W2_m2)
        return O0, O1, O2

    # forward rows of the sampled atoms: every edge into them
    Dd = d["dst_in_s"]
    xe_o, wig_o, env_o = _oracle_geometry(d, Dd)
    xn = (c["x"] * 0.7).double()
    O = edge_msgs(Dd, xn, xe_o, wig_o, env_o)
    ref = oops.rotate_scatter_split(*O, wig_o, env_o, c["x"].double(), c["idx_j"][Dd], None, None, N2)
    assert _rel(out[S.to(DEV)], ref[S]) < 2e-5

    # node gradient on the sampled atoms: every edge touching them; edge gradients on the sample
    T = torch.unique(torch.cat([d["touch_s"], Es]))
    xe_o, wig_o, env_o = _oracle_geometry(d, T)
    xn = (c["x"] * 0.7).double().requires_grad_(True)
    xi = c["x"].double().requires_grad_(True)
    xgo = xe_o[:, :B2].clone().requires_grad_(True)
    wo, eo = wig_o.clone().requires_grad_(True), env_o.clone().requires_grad_(True)
    O = edge_msgs(T, xn, torch.cat([xgo, xe_o[:, B2:]], 1), wo, eo)
    ref = oops.rotate_scatter_split(*O, wo, eo, xi, c["idx_j"][T], None, None, N2)
    gxn_o, gxi_o, gg_o, gw_o, ge_o = torch.autograd.grad(ref, [xn, xi, xgo, wo, eo], gmid.double())
    assert _rel(gxn[S.to(DEV)], gxn_o[S]) < 5e-5
    assert _rel(gxi[S.to(DEV)], gxi_o[S]) < 2e-5
    pos = torch.searchsorted(T, Es)
    assert _rel(gw[Es.to(DEV)], gw_o[pos]) < 5e-5
    assert _rel(ge[Es.to(DEV)], ge_o[pos]) < 5e-5
    assert _rel(gg[Es.to(DEV)], gg_o[pos]) < 5e-5


def test_config3_f16_mode_tf32_accuracy_class():
    """The single-product "f16" mode (16-bit storage of the per-edge GEMM results, one fp16
    product per GEMM) on the full config-3 system, against the default f16x3 path (itself held to
    the fp64 oracle above): within the TF32 accuracy class (energy 1e-3 relative, forces
    1e-2 eV/A; the reference's own TF32 path deviates 2e-2 eV/A on this system), no fp16 range
    error at this size, and bitwise reproducible run to run."""
    from flash_uma_b200.linear import check_errors
    from flash_uma_b200.predict import Predictor
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
    from flash_uma_b200.systems import config3_system, to_graph
    from flash_uma_b200.wrapper import ZeroAllocBackbone
    data = to_graph([config3_system()]).to(DEV)
    off = SyntheticESCNMDBackbone(seed=0)
    head = make_energy_head(128, 128, seed=1).to(DEV)
    out = {}
    for gemm in ("f16x3", "f16"):
        bb = ZeroAllocBackbone(copy.deepcopy(off).to(DEV), gemm=gemm)
        pred = Predictor(bb, head)
        out[gemm] = [pred(data) for _ in range(2)]
    torch.cuda.synchronize()
    check_errors()
    a, b = out["f16"]
    assert torch.equal(a["energy"], b["energy"]) and torch.equal(a["forces"], b["forces"])
    ref = out["f16x3"][0]
    erel = ((a["energy"].double() - ref["energy"].double()).abs() / ref["energy"].double().abs()).max().item()
    ferr = (a["forces"].double() - ref["forces"].double()).abs().max().item()
    assert erel < 1e-3, erel
    assert ferr < 1e-2, ferr
