"""GPU parity: every registry geometry against the CPU oracle, through the C ABI.

Tolerances (stated here, checked per element), relative error |a - e| / (|e| + atol):
* fp16 h against the oracle's h: atol = 1e-3 * max|h|, bound 1e-2; every element
  within one fp16 ulp plus the fp32 summation bound carried through the
  activation, |dh/dg| * K * 2^-24 * sum|Wg x| + |dh/du| * K * 2^-24 * sum|Wu x|;
  and at most 2% of the elements with other bits (the GPU sums in fp32, the oracle
  in double, so a value near an fp16 rounding midpoint can round the other way;
  truncating instead of rounding to nearest would change about half);
* fp32 y against the oracle's down projection of the GPU's own h:
  atol_j = 2^-11 * sum_i |Wd[j,i] * h[i]|, bound 2e-3 (checking y against the
  oracle's h instead would charge one flipped h element, |Wd[j,i]| * ulp(h_i), to
  every row j);
* and y against the full oracle with the reference's own gate
  (include/contract.hpp:36-53): atol 0.003, rtol 0.01.
The model-rounding binding path is checked as tools/gpu_validate.py checks it
(torch fp16 reference, atol .01, rtol .02) and against the oracle's fp16 path.
"""
import numpy as np
import pytest
import torch

import oracle as O
from swiglu_b200 import binding
from swiglu_b200.binding import config_ids

pytestmark = pytest.mark.gpu

H_TOL = 1e-2
Y_TOL = 2e-3

CORRECTNESS = [(1, 1), (37, 65), (129, 257), (512, 1024), (1, 9), (2, 3), (8, 8), (7, 9), (9, 7), (31, 33),
               (32, 32), (33, 31), (64, 64), (66, 70), (256, 256), (264, 272), (1024, 256), (1025, 513),
               (1030, 514)]
BASELINE_SHAPES = [(17, 33), (2047, 5631), (2048, 5632), (2048, 8192), (4096, 11008), (4096, 14336)]


def rel_err(actual, expected, atol=None):
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    if atol is None:
        atol = 1e-3 * max(float(np.max(np.abs(e))), 1e-30)
    return float(np.max(np.abs(a - e) / (np.abs(e) + atol)))


def y_atol(wd, h):
    """Per-row error scale of y from one fp16 rounding of h: 2^-11 * sum_i |Wd[j,i] h[i]|."""
    return 2.0 ** -11 * (np.abs(wd.astype(np.float32)) @ np.abs(h.astype(np.float32))).astype(np.float64)


def h_bound(w, e):
    """One fp16 ulp of the oracle's h plus the fp32 summation bound carried through silu(g) * u."""
    f = lambda a: O.f16_values(a).astype(np.float64)  # noqa: E731
    x = f(w["x"])
    wg, wu = f(w["wg"]), f(w["wu"])
    g, u = wg @ x + f(w["bg"]), wu @ x + f(w["bu"])
    gamma = x.size * 2.0 ** -24
    sig = 1.0 / (1.0 + np.exp(-g))
    dg = np.abs(sig * (1 + g * (1 - sig)) * u)  # d(silu(g) u)/dg
    return (np.spacing(np.abs(e)).astype(np.float64) + 1e-12
            + gamma * (dg * (np.abs(wg) @ np.abs(x)) + np.abs(g * sig) * (np.abs(wu) @ np.abs(x))))


def check_h_close(h, case):
    """Per-element bound (one ulp + fp32 summation error), at most 2% of bits off, and the relative bound."""
    h = np.asarray(h, np.float16)
    e = np.asarray(case.act, np.float16)
    assert np.isfinite(h.astype(np.float32)).all()
    if getattr(case, "_h_bound", None) is None:
        case._h_bound = h_bound(case.w, e)
    bound = case._h_bound
    diff = np.abs(h.astype(np.float64) - e.astype(np.float64))
    assert (diff <= bound).all(), int(np.argmax(diff - bound))
    assert np.mean(h.view(np.uint16) != e.view(np.uint16)) <= 0.02
    assert rel_err(h, e) <= H_TOL


def check_y_given_h(w, h_gpu, y_gpu, y_full):
    """y against the oracle's down projection of the GPU's h, then against the full oracle (reference gate)."""
    h16 = np.asarray(h_gpu, np.float16)
    y_own = O.project(w["wd"], h16, w["bd"], w["x"])
    assert rel_err(y_gpu, y_own, y_atol(w["wd"], h16)) <= Y_TOL
    assert O.compare(y_gpu, y_full)[0]


def dev(a, offset=0):
    """Upload a float16/float32 numpy array; offset>0 places it `offset` elements past an aligned start."""
    t = torch.from_numpy(np.ascontiguousarray(a))
    if offset:
        backing = torch.empty(t.numel() + offset, dtype=t.dtype, device="cuda")
        out = backing[offset:].view(t.shape)
        out.copy_(t)
        return out
    return t.cuda()


class Case:
    def __init__(self, hidden, inter, dist="normal", x_offset=0, w_offset=0):
        self.hidden, self.inter = hidden, inter
        w = O.normal_workload(0, hidden, inter) if dist == "normal" else O.reference_workload(17, hidden, inter)
        self.w = w
        self.proj, self.act, self.y = O.ffn(w)
        self.d = {k: dev(v, w_offset if k in ("wg", "wu", "wd") else (x_offset if k == "x" else 0))
                  for k, v in w.items()}
        self.act_d = dev(self.act)
        # down-kernel reference on the oracle's own h: isolates the down kernel
        self.y_down = O.project(w["wd"], self.act, w["bd"], w["x"])
        self.y_atol = y_atol(w["wd"], self.act)

    def gate(self, cfg):
        h = torch.empty(self.inter, dtype=torch.float16, device="cuda")
        d = self.d
        binding.gate(d["wg"], d["wu"], d["x"], h, cfg, d["bg"], d["bu"])
        return h

    def down(self, cfg):
        y = torch.empty(self.hidden, dtype=torch.float32, device="cuda")
        binding.project(self.d["wd"], self.act_d, y, cfg, bias=self.d["bd"], residual=self.d["x"])
        return y


def check_gate(case, h):
    check_h_close(h.cpu().numpy(), case)


def check_down(case, y):
    y = y.cpu().numpy()
    assert rel_err(y, case.y_down, case.y_atol) <= Y_TOL
    assert O.compare(y, case.y_down)[0]


@pytest.fixture(scope="module")
def ids():
    return config_ids()


@pytest.mark.parametrize("shape", CORRECTNESS)
def test_correctness_suite_every_config(shape, ids):
    case = Case(*shape, dist="uniform")
    for cfg in ids:
        check_gate(case, case.gate(cfg))
        check_down(case, case.down(cfg))
    torch.cuda.synchronize()
    assert binding.device_error() == 0


@pytest.mark.parametrize("shape", BASELINE_SHAPES)
def test_baseline_shapes_every_config(shape, ids):
    case = Case(*shape)
    for cfg in ids:
        check_gate(case, case.gate(cfg))
        check_down(case, case.down(cfg))
    assert binding.device_error() == 0


@pytest.mark.parametrize("shape,x_off,w_off", [((2048, 5632), 1, 0), ((2047, 5631), 1, 0), ((17, 33), 1, 0),
                                               ((256, 264), 0, 1), ((2048, 5632), 1, 1), ((66, 70), 3, 5)])
def test_misaligned_inputs_every_config(shape, x_off, w_off, ids):
    case = Case(*shape, x_offset=x_off, w_offset=w_off)
    assert case.d["x"].data_ptr() % 16 != 0 or x_off == 0
    for cfg in ids:
        check_gate(case, case.gate(cfg))
        check_down(case, case.down(cfg))


@pytest.mark.parametrize("shape", [(37, 65), (2048, 5632), (4096, 14336)])
def test_full_layer_matches_reference_oracle(shape, ids):
    case = Case(*shape)
    d = case.d
    pairs = [(g, dd) for g in ids for dd in ids if g == dd or {g, dd} & {33, 64, 65}]
    for g, dd in pairs:
        h = torch.empty(case.inter, dtype=torch.float16, device="cuda")
        y = torch.empty(case.hidden, dtype=torch.float32, device="cuda")
        binding.ffn(d["x"], d["wg"], d["wu"], d["wd"], d["bg"], d["bu"], d["bd"], h, y, g, dd)
        hc = h.cpu().numpy()
        check_h_close(hc, case)
        check_y_given_h(case.w, hc, y.cpu().numpy(), case.y)


def test_reference_golden_uniform_workload(ids):
    """The reference's own seed-17 workload: y within the reference's gate of its stored outputs."""
    data = np.load(O.HERE.parent / "tests" / "golden" / "reference_small.npz")
    names = sorted({k.split("/")[0] for k in data.files})
    for name in names:
        w = {k: data[f"{name}/{k}"].view(np.float16) for k in ("wg", "wu", "wd", "x", "bg", "bu", "bd")}
        d = {k: dev(v) for k, v in w.items()}
        inter, hidden = w["wg"].shape
        for cfg in (1, 16, 33, 64):
            h = torch.empty(inter, dtype=torch.float16, device="cuda")
            y = torch.empty(hidden, dtype=torch.float32, device="cuda")
            binding.ffn(d["x"], d["wg"], d["wu"], d["wd"], d["bg"], d["bu"], d["bd"], h, y, cfg, cfg)
            assert O.compare(y.cpu().numpy(), data[f"{name}/y"])[0], (name, cfg)


def test_raw_projection_fp32(ids):
    case = Case(2048, 8192)
    for cfg in ids:
        g = torch.empty(8192, dtype=torch.float32, device="cuda")
        binding.project(case.d["wg"], case.d["x"], g, cfg)
        gc = g.cpu().numpy()
        # fp32 projection: error scale 2^-11 * sum |W x| (fp16 inputs, fp32 accumulation)
        assert rel_err(gc, case.proj, y_atol(case.w["wg"], case.w["x"])) <= Y_TOL
        assert O.compare(gc, case.proj)[0]


def test_half_output_projection(ids):
    case = Case(512, 1024)
    expect = O.project(case.w["wd"], case.act, half_out=True)
    for cfg in ids:
        out = torch.empty(512, dtype=torch.float16, device="cuda")
        binding.project(case.d["wd"], case.act_d, out, cfg)
        assert rel_err(out.cpu().numpy(), expect) <= H_TOL


def test_deterministic_across_runs(ids):
    case = Case(4096, 11008)
    for cfg in ids:
        a, b = case.gate(cfg), case.gate(cfg)
        assert torch.equal(a, b)
        ya, yb = case.down(cfg), case.down(cfg)
        assert torch.equal(ya, yb)


# ---- the drop-in binding (tools/gpu_validate.py semantics) --------------------

@pytest.mark.parametrize("hidden,inter", [(1, 1), (7, 9), (8, 8), (31, 33), (64, 70), (256, 264), (513, 1025)])
def test_binding_every_pair_aligned_and_misaligned(hidden, inter, ids):
    torch.manual_seed(101)
    with torch.inference_mode():
        weights = [torch.randn((inter, hidden), device="cuda", dtype=torch.float16) / hidden ** .5,
                   torch.randn((inter, hidden), device="cuda", dtype=torch.float16) / hidden ** .5,
                   torch.randn((hidden, inter), device="cuda", dtype=torch.float16) / inter ** .5]
        for offset in (0, 1):
            backing = torch.randn((hidden + offset,), device="cuda", dtype=torch.float16)
            x = backing[offset:].view(1, 1, hidden)
            expected = (torch.nn.functional.silu(x @ weights[0].T) * (x @ weights[1].T)) @ weights[2].T
            h = torch.empty((inter,), device="cuda", dtype=torch.float16)
            y = torch.empty_like(x)
            for g in ids:
                for d in ids:
                    binding.swiglu_out(x, *weights, h, y, g, d)
                    torch.testing.assert_close(y, expected, atol=.01, rtol=.02)
            with pytest.raises(RuntimeError, match="workspace overlaps input storage"):
                binding.swiglu_out(x, *weights, h, x, 1, 1)
            for invalid in (0, 999, 2 ** 32 + 1):
                with pytest.raises(RuntimeError):
                    binding.swiglu_out(x, *weights, h, y, invalid, 1)


def test_binding_matches_oracle_model_rounding(ids):
    w = O.normal_workload(4, 2048, 5632)
    h_ref, y_ref = O.ffn_model(w)
    d = {k: dev(v) for k, v in w.items()}
    x = d["x"].view(1, 1, -1)
    h = torch.empty(5632, dtype=torch.float16, device="cuda")
    y = torch.empty_like(x)
    for cfg in ids:
        binding.swiglu_out(x, d["wg"], d["wu"], d["wd"], h, y, cfg, cfg)
        hc = h.cpu().numpy()
        # fp16 rounding points match; differences are at most a couple of ulps
        assert rel_err(hc, h_ref) <= H_TOL
        assert np.mean(hc.view(np.uint16) == h_ref.view(np.uint16)) > 0.97
        assert rel_err(y.cpu().numpy().ravel(), y_ref) <= H_TOL


def test_swiglu_allocating_wrapper():
    w = O.normal_workload(5, 256, 512)
    d = {k: dev(v) for k, v in w.items()}
    x = d["x"].view(1, 1, -1)
    y1 = binding.swiglu(x, d["wg"], d["wu"], d["wd"], 33)
    h = torch.empty(512, dtype=torch.float16, device="cuda")
    y2 = torch.empty_like(x)
    binding.swiglu_out(x, d["wg"], d["wu"], d["wd"], h, y2, 33, 33)
    assert torch.equal(y1, y2)


def test_binding_inside_cuda_graph():
    w = O.normal_workload(6, 2048, 5632)
    d = {k: dev(v) for k, v in w.items()}
    x = d["x"].view(1, 1, -1)
    h = torch.empty(5632, dtype=torch.float16, device="cuda")
    y = torch.empty_like(x)
    for cfg in (16, 33, 64):
        binding.swiglu_out(x, d["wg"], d["wu"], d["wd"], h, y, cfg, cfg)
        eager = y.clone()
        y.zero_()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            binding.swiglu_out(x, d["wg"], d["wu"], d["wd"], h, y, cfg, cfg)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(y, eager)


def test_cublas_baseline_matches_oracle():
    case = Case(2048, 5632)
    d = case.d
    base = binding.CublasBaseline()
    g = torch.empty(5632, dtype=torch.float32, device="cuda")
    u = torch.empty_like(g)
    h = torch.empty(5632, dtype=torch.float16, device="cuda")
    y = torch.empty(2048, dtype=torch.float32, device="cuda")
    for algo in (0, 1):
        base.ffn(d["x"], d["wg"], d["wu"], d["wd"], d["bg"], d["bu"], d["bd"], g, u, h, y, algo=algo)
        assert O.compare(y.cpu().numpy(), case.y)[0]
        assert rel_err(h.cpu().numpy(), case.act) <= H_TOL
    base.close()


# ---- the fused whole-layer kernel (one persistent launch) --------------------

@pytest.mark.parametrize("shape", [(4096, 14336), (4096, 11008), (2048, 8192), (2048, 5632), (512, 1376),
                                   (64, 96), (1024, 256)])
def test_fused_layer_kernel_matches_oracle(shape):
    case = Case(*shape)
    d = case.d
    ws = binding.layer_workspace()
    for cfg in binding.layer_config_ids():
        for _ in range(2):  # the launch epoch advances call after call
            h = torch.empty(case.inter, dtype=torch.float16, device="cuda")
            y = torch.empty(case.hidden, dtype=torch.float32, device="cuda")
            binding.ffn_fused(d["x"], d["wg"], d["wu"], d["wd"], d["bg"], d["bu"], d["bd"], h, y, cfg, ws)
            hc = h.cpu().numpy()
            check_h_close(hc, case)
            check_y_given_h(case.w, hc, y.cpu().numpy(), case.y)
    assert binding.device_error() == 0


@pytest.mark.parametrize("layer", [220, 221, 223])
def test_streaming_layer_chain_matches_plain_calls(layer):
    """Streaming whole-layer kernels chained with SWB_PREFETCH_WEIGHTS (each launched
    programmatically, its weight stream starting while the previous layer still runs) give
    bit-identical outputs to plain (cooperative) calls, eagerly and in one CUDA graph, and the
    workspace's block words come back to zero after every call."""
    H, I = 4096, 14336
    d = [{k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in O.normal_workload(seed, H, I).items()}
         for seed in (0, 1)]
    ws = binding.layer_workspace()
    h = torch.empty(I, dtype=torch.float16, device="cuda")
    ref = []
    for k in range(2):
        y = torch.empty(H, dtype=torch.float32, device="cuda")
        binding.ffn_fused(d[k]["x"], d[k]["wg"], d[k]["wu"], d[k]["wd"], d[k]["bg"], d[k]["bu"], d[k]["bd"], h, y,
                          layer, ws)
        torch.cuda.synchronize()
        ref.append(y.clone())
    ys = [torch.empty(H, dtype=torch.float32, device="cuda") for _ in range(6)]
    stream = torch.cuda.Stream()

    def chain():
        for k in range(6):
            w = d[k % 2]
            binding.ffn_fused(w["x"], w["wg"], w["wu"], w["wd"], w["bg"], w["bu"], w["bd"], h, ys[k], layer, ws,
                              stream=stream.cuda_stream, prefetch_weights=True)

    with torch.cuda.stream(stream):
        chain()
        stream.synchronize()
        assert all(torch.equal(ys[k], ref[k % 2]) for k in range(6))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            chain()
        for _ in range(3):
            for yk in ys:
                yk.zero_()
            g.replay()
            stream.synchronize()
            assert all(torch.equal(ys[k], ref[k % 2]) for k in range(6))
        g.reset()
    torch.cuda.synchronize()
    assert int(ws.view(torch.int32)[1:].abs().sum()) == 0  # done counter and block words reset
    assert binding.device_error() == 0


@pytest.mark.parametrize("gcfg,dcfg", [(69, 87), (33, 35), (82, 82), (96, 87)])
def test_prefetch_chain_matches_plain_calls(gcfg, dcfg):
    """Layers chained back to back with SWB_PREFETCH_WEIGHTS (each gate starts streaming its
    weights while the previous layer's down kernel still runs; x, h touched only after it
    completes) give bit-identical outputs to plain calls, eagerly and in one CUDA graph."""
    H, I = 2048, 5632
    d = [{k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in O.normal_workload(seed, H, I).items()}
         for seed in (0, 1)]
    h = torch.empty(I, dtype=torch.float16, device="cuda")
    ref = []
    for k in range(2):
        y = torch.empty(H, dtype=torch.float32, device="cuda")
        binding.ffn(d[k]["x"], d[k]["wg"], d[k]["wu"], d[k]["wd"], d[k]["bg"], d[k]["bu"], d[k]["bd"], h, y, gcfg, dcfg)
        torch.cuda.synchronize()
        ref.append(y.clone())
    ys = [torch.empty(H, dtype=torch.float32, device="cuda") for _ in range(4)]
    stream = torch.cuda.Stream()

    def chain():
        for k in range(4):
            w = d[k % 2]
            binding.ffn(w["x"], w["wg"], w["wu"], w["wd"], w["bg"], w["bu"], w["bd"], h, ys[k], gcfg, dcfg,
                        stream=stream.cuda_stream, prefetch_weights=True)

    with torch.cuda.stream(stream):
        chain()
        stream.synchronize()
        for k in range(4):
            assert torch.equal(ys[k], ref[k % 2]), k
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            chain()
        for _ in range(3):
            for yk in ys:
                yk.zero_()
            g.replay()
            stream.synchronize()
            for k in range(4):
                assert torch.equal(ys[k], ref[k % 2]), k
        g.reset()
    assert binding.device_error() == 0


PAD = 256
SENTINEL = {torch.float16: -1234.0, torch.float32: -98765.0}


def guarded(n, dtype):
    """A length-n output inside a buffer whose PAD elements on each side hold a sentinel."""
    buf = torch.full((n + 2 * PAD,), SENTINEL[dtype], dtype=dtype, device="cuda")
    return buf, buf[PAD:PAD + n]


def pads_intact(buf):
    s = SENTINEL[buf.dtype]
    return bool(torch.all(buf[:PAD] == s).item()) and bool(torch.all(buf[-PAD:] == s).item())


@pytest.mark.parametrize("shape", [(17, 33), (37, 65), (2047, 5631), (4096, 1792)])
def test_outputs_stay_in_their_bounds(shape, ids):
    """Guard-band canaries: every geometry writes exactly its output elements (gate h, fp32
    and fp16 projections, the layer, the fused single-rank exchange, the fused layer kernel),
    at odd sizes and tensor-parallel shard sizes; the sentinel pads either side survive."""
    from swiglu_b200 import tp as T
    H, I = shape
    g = torch.Generator(device="cuda").manual_seed(5)
    r = lambda *sz: (torch.randn(*sz, generator=g, device="cuda") * 0.05).half()  # noqa: E731
    wg, wu, wd, x, bg, bu, bd = r(I, H), r(I, H), r(H, I), r(H), r(I), r(I), r(H)
    for cfg in ids:
        hb, h = guarded(I, torch.float16)
        binding.gate(wg, wu, x, h, cfg, bg, bu)
        yb, y = guarded(H, torch.float32)
        binding.project(wd, h, y, cfg, bias=bd, residual=x)
        yhb, yh = guarded(H, torch.float16)
        binding.project(wd, h, yh, cfg)
        hb2, h2 = guarded(I, torch.float16)
        yb2, y2 = guarded(H, torch.float32)
        binding.ffn(x, wg, wu, wd, bg, bu, bd, h2, y2, cfg, cfg)
        torch.cuda.synchronize()
        assert all(pads_intact(b) for b in (hb, yb, yhb, hb2, yb2)), cfg
    if H % 8 == 0 and I % 8 == 0:
        ex = T.Exchange(0, 1, H, torch.device("cuda", 0))
        s = {"wg": wg, "wu": wu, "wd": wd, "bg": bg, "bu": bu}
        for gate_cfg, down_cfg in ((69, 87), (33, 83), (82, 80)) + tuple((lid, 0) for lid in binding.layer_config_ids()):
            hb, h = guarded(I, torch.float16)
            yb, y = guarded(H, torch.float32)
            T.ffn_tp_fused(ex, x, s, bd, h, y, gate_cfg, down_cfg)
            torch.cuda.synchronize()
            assert pads_intact(hb) and pads_intact(yb), (gate_cfg, down_cfg)
        ex.close()
        ws = binding.layer_workspace()
        for lid in binding.layer_config_ids():
            hb, h = guarded(I, torch.float16)
            yb, y = guarded(H, torch.float32)
            binding.ffn_fused(x, wg, wu, wd, bg, bu, bd, h, y, lid, ws)
            torch.cuda.synchronize()
            assert pads_intact(hb) and pads_intact(yb), lid
    assert binding.device_error() == 0


def test_fused_layer_in_cuda_graph_and_unsupported_shapes():
    case = Case(2048, 5632)
    d = case.d
    ws = binding.layer_workspace()
    h = torch.empty(case.inter, dtype=torch.float16, device="cuda")
    y = torch.empty(case.hidden, dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        binding.ffn_fused(d["x"], d["wg"], d["wu"], d["wd"], d["bg"], d["bu"], d["bd"], h, y, 200, ws)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            binding.ffn_fused(d["x"], d["wg"], d["wu"], d["wd"], d["bg"], d["bu"], d["bd"], h, y, 200, ws)
        for _ in range(4):
            y.zero_()
            g.replay()
            torch.cuda.synchronize()
            check_y_given_h(case.w, h.cpu().numpy(), y.cpu().numpy(), case.y)
        g.reset()
    odd = Case(2047, 5631)
    with pytest.raises(RuntimeError, match="unsupported"):
        binding.ffn_fused(odd.d["x"], odd.d["wg"], odd.d["wu"], odd.d["wd"], odd.d["bg"], odd.d["bu"], odd.d["bd"],
                          torch.empty(5631, dtype=torch.float16, device="cuda"),
                          torch.empty(2047, dtype=torch.float32, device="cuda"), 200, ws)
    assert binding.device_error() == 0
