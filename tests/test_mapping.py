"""Host simulation of every kernel's thread -> element mapping (no GPU).

Extends the reference's address-coverage audit (tests/mapping_tests.cpp:6-27:
every column read exactly once, every output row written exactly once, for all
configs x correctness shapes x both orientations x input offsets {0,2,4,8} bytes)
to this build's kernels:

* ldg_kernel: scalar head up to the first aligned weight, vector body with
  UNROLL loads in flight, scalar tail; every vector load aligned;
* bulk_kernel: balanced row ranges per CTA, chunked cp.async.bulk copies whose
  sizes and addresses are 16-byte multiples and whose expect_tx totals equal the
  bytes copied, ring-stage reuse order, shared-memory layout within 227 KB.

The index arithmetic below restates cuda-kernel_b200/csrc/kernels.cuh and the
launch arithmetic of csrc/swiglu_b200.cu line by line.
"""
import math

import numpy as np
import pytest

from swiglu_b200 import config_ids, config_info

CORRECTNESS = [(1, 1), (37, 65), (129, 257), (512, 1024), (1, 9), (2, 3), (8, 8), (7, 9), (9, 7), (31, 33),
               (32, 32), (33, 31), (64, 64), (66, 70), (256, 256), (264, 272), (1024, 256), (1025, 513),
               (1030, 514)]
EXTRA = [(17, 33), (2047, 5631), (2048, 5632), (4096, 14336)]
SMEM_PER_SM = 233472
SMEM_PER_CTA = 232448
SMS = 148


def ldg_row_coverage(T, pack, unroll, cols, w_addr, u_addr=None):
    """Columns touched by the T threads of one row; returns (counts, vector addresses)."""
    VB = 2 * pack
    vec = True
    if u_addr is not None:
        vec = (u_addr - w_addr) % VB == 0
    peel = ((VB - w_addr % VB) % VB) // 2 if vec else cols
    peel = min(peel, cols)
    nvec = (cols - peel) // pack
    tail0 = peel + nvec * pack
    counts = np.zeros(cols, np.int64)
    addrs = []
    for t in range(T):
        for c in range(t, peel, T):
            counts[c] += 1
        v = t
        while v + (unroll - 1) * T < nvec:
            for i in range(unroll):
                c = peel + (v + i * T) * pack
                counts[c:c + pack] += 1
                addrs.append(w_addr + 2 * c)
            v += unroll * T
        while v < nvec:
            c = peel + v * pack
            counts[c:c + pack] += 1
            addrs.append(w_addr + 2 * c)
            v += T
        for c in range(tail0 + t, cols, T):
            counts[c] += 1
    return counts, addrs, peel, VB


def audit_ldg(cfg, rows, cols, offset_bytes, gated):
    W, R, pack, unroll = cfg["warps"], cfg["rows"], cfg["pack"], cfg["unroll"]
    T = 32 * W
    base = 4096 + offset_bytes
    seen_peels = {}
    for row in range(rows):
        w_addr = base + 2 * row * cols
        u_addr = (1 << 30) + offset_bytes + 2 * row * cols if gated else None
        key = (w_addr % 16, None if u_addr is None else u_addr % 16)
        if key in seen_peels:
            continue
        counts, addrs, peel, VB = ldg_row_coverage(T, pack, unroll, cols, w_addr, u_addr)
        assert (counts == 1).all(), ("column omitted or duplicated", cfg["id"], rows, cols, offset_bytes)
        assert all(a % VB == 0 for a in addrs), "misaligned vector load"
        # staged-x vector reads start on 16-byte (pack 8) / 8-byte (pack 2) boundaries when enabled
        seen_peels[key] = peel
    grid = (rows + R - 1) // R
    outputs = np.zeros(rows, np.int64)
    for block in range(grid):
        for warp in range(W * R):
            group, sub = warp // W, warp % W
            row = block * R + group
            if sub == 0 and row < rows:
                outputs[row] += 1
    assert (outputs == 1).all(), "output omitted or duplicated"


def bulk_layout(nm, chunk, stages, cols, cw, rows_per_cta):
    def up(v, a):
        return (v + a - 1) // a * a
    ring = stages * nm * chunk * 2
    full = up(ring, 16)
    empty = full + stages * 8
    xs = up(empty + stages * 8, 16)
    part = up(xs + cols * 4, 16)
    total = up(part + rows_per_cta * cw * nm * 4, 16)
    return {"ring": 0, "full": full, "empty": empty, "xs": xs, "part": part, "total": total}


def bulk_plan(cfg, rows, cols, gated, w_aligned=True):
    """Mirror of launch_bulk: returns None when the fallback geometry runs."""
    nm = 2 if gated else 1
    cw, cps, chunk, smax = cfg["warps"], cfg["rows"], cfg["chunk"], cfg["stages"]
    G = min(SMS * cps, rows)
    rpc = (rows + G - 1) // G
    budget = min(SMEM_PER_CTA, SMEM_PER_SM // cps - 1024) - 64
    stages = smax
    while stages >= 2 and bulk_layout(nm, chunk, stages, cols, cw, rpc)["total"] > budget:
        stages -= 1
    if cols % 8 or not w_aligned or stages < 2:
        return None
    return {"G": G, "rpc": rpc, "stages": stages, "layout": bulk_layout(nm, chunk, stages, cols, cw, rpc),
            "budget": budget}


def audit_bulk(cfg, rows, cols, gated):
    plan = bulk_plan(cfg, rows, cols, gated)
    if plan is None:
        return False
    nm = 2 if gated else 1
    cw, chunk = cfg["warps"], cfg["chunk"]
    CT = cw * 32
    G, stages, L = plan["G"], plan["stages"], plan["layout"]
    assert L["total"] <= plan["budget"]
    assert L["full"] % 8 == 0 and L["empty"] % 8 == 0 and L["xs"] % 16 == 0
    assert (nm * chunk * 2) % 16 == 0
    row_owner = np.zeros(rows, np.int64)
    nch = (cols + chunk - 1) // chunk
    for b in range(G):
        r0, r1 = (b * rows) // G, ((b + 1) * rows) // G
        assert r1 - r0 >= 1 and r1 - r0 <= plan["rpc"]
        row_owner[r0:r1] += 1
        units = (r1 - r0) * nch
        # producer: stage reuse order, byte counts, alignment
        fills = {}
        row, ch = r0, 0
        for k in range(units):
            s = k % stages
            if k >= stages:
                assert fills[s] == k - stages  # the consumer release waited for is this stage's previous fill
            fills[s] = k
            c0 = ch * chunk
            length = min(chunk, cols - c0)
            nbytes = length * 2
            assert nbytes % 16 == 0 and nbytes > 0
            src = 2 * (row * cols + c0)
            assert src % 16 == 0
            dst = s * nm * chunk * 2
            assert dst % 16 == 0 and dst + nm * nbytes <= L["full"]
            assert nbytes * nm < (1 << 20)  # mbarrier tx-count range
            ch += 1
            if ch == nch:
                ch, row = 0, row + 1
        assert row == r1
        # consumer: every column of a chunk read by exactly one thread
        for c0 in range(0, cols, chunk):
            nv = min(chunk, cols - c0) // 8
            counts = np.zeros(nv, np.int64)
            for t in range(CT):
                counts[t:nv:CT] += 1
            assert (counts == 1).all()
        if b > 3 and b < G - 3:
            continue
    assert (row_owner == 1).all()
    return True


def rbulk_layout(nm, rs, cols, stages, cw, rows_per_cta):
    def up(v, a):
        return (v + a - 1) // a * a
    full = up(stages * rs * nm * cols * 2, 16)
    empty = full + stages * 8
    part = up(empty + stages * 8, 16)
    return {"full": full, "empty": empty, "part": part, "total": up(part + rows_per_cta * cw * nm * 4, 16)}


def rbulk_plan(cfg, rows, cols, gated, w_aligned=True):
    """Mirror of launch_rbulk: None when the fallback geometry runs."""
    nm = 2 if gated else 1
    cw, cps, maxj, target, smax = cfg["warps"], cfg["rows"], cfg["unroll"], cfg["chunk"], cfg["stages"]
    nv = cols // 8
    ok = cols % 8 == 0 and w_aligned and nv <= maxj * cw * 32
    G = min(SMS * cps, rows)
    rpc = (rows + G - 1) // G
    budget = min(SMEM_PER_CTA, SMEM_PER_SM // cps - 1024) - 64
    row_bytes = nm * cols * 2
    rs = min(max(1, target // max(row_bytes, 1)), rpc)
    stages = 0
    while rs >= 1:
        stages = smax
        while stages >= 2 and rbulk_layout(nm, rs, cols, stages, cw, rpc)["total"] > budget:
            stages -= 1
        if stages >= 2 or rs == 1:
            break
        rs = rs // 2 if rs > 1 else 0
    if not ok or rs < 1 or stages < 2:
        return None
    stages = min(stages, max(2, (rpc + rs - 1) // rs))  # no deeper than a CTA's stages of work
    return {"G": G, "rpc": rpc, "rs": rs, "stages": stages, "budget": budget,
            "layout": rbulk_layout(nm, rs, cols, stages, cw, rpc)}


def audit_rbulk(cfg, rows, cols, gated):
    plan = rbulk_plan(cfg, rows, cols, gated)
    if plan is None:
        return False
    nm = 2 if gated else 1
    CT = cfg["warps"] * 32
    nv = cols // 8
    G, rs, stages, L = plan["G"], plan["rs"], plan["stages"], plan["layout"]
    assert L["total"] <= plan["budget"] and L["full"] % 16 == 0 and L["part"] % 16 == 0
    # consumer ownership of a row's vectors: t + j*CT for j < MAXJ covers [0, nv) once
    counts = np.zeros(nv, np.int64)
    for t in range(CT):
        for j in range(cfg["unroll"]):
            v = t + j * CT
            if v < nv:
                counts[v] += 1
    assert (counts == 1).all()
    owner = np.zeros(rows, np.int64)
    stage_bytes = rs * nm * cols * 2
    for b in range(G):
        r0, r1 = (b * rows) // G, ((b + 1) * rows) // G
        assert 1 <= r1 - r0 <= plan["rpc"]
        units = (r1 - r0 + rs - 1) // rs
        covered = 0
        for k in range(units):
            s = k % stages
            row = r0 + k * rs
            ru = min(rs, r1 - row)
            nbytes = ru * cols * 2
            assert nbytes % 16 == 0 and (2 * row * cols) % 16 == 0
            assert s * stage_bytes % 16 == 0 and s * stage_bytes + nm * rs * cols * 2 <= L["full"]
            assert nbytes * nm < (1 << 20)
            owner[row:row + ru] += 1
            covered += ru
        assert covered == r1 - r0
    assert (owner == 1).all()
    return True


@pytest.fixture(scope="module")
def configs():
    return [config_info(i) for i in config_ids()]


@pytest.mark.parametrize("shape", CORRECTNESS)
def test_ldg_coverage(configs, shape):
    h, i = shape
    n = 0
    for cfg in configs:
        if cfg["family"] != 0:
            continue
        for off in (0, 2, 4, 8):
            for rows, cols in ((i, h), (h, i)):
                for gated in (True, False):
                    audit_ldg(cfg, rows, cols, off, gated)
                    n += 1
    assert n > 0


@pytest.mark.parametrize("shape", CORRECTNESS + EXTRA)
def test_bulk_plan_and_coverage(configs, shape):
    h, i = shape
    for cfg in configs:
        if cfg["family"] != 1:
            continue
        for rows, cols, gated in ((i, h, True), (h, i, False)):
            ran = audit_bulk(cfg, rows, cols, gated)
            if cols % 8 == 0 and cols <= 16384:
                assert ran, (cfg["id"], rows, cols)


def test_bulk_large_shapes_fit_every_geometry(configs):
    for cfg in configs:
        if cfg["family"] != 1:
            continue
        for rows, cols, gated in ((14336, 4096, True), (4096, 14336, False), (11008, 4096, True),
                                  (4096, 11008, False), (5632, 2048, True), (2048, 5632, False)):
            plan = bulk_plan(cfg, rows, cols, gated)
            assert plan is not None and plan["stages"] >= 2, (cfg["id"], rows, cols)
            # one CTA per SM set, rows balanced within one row
            per = [((b + 1) * rows) // plan["G"] - (b * rows) // plan["G"] for b in range(plan["G"])]
            assert max(per) - min(per) <= 1


def test_bulk_falls_back_when_unaligned(configs):
    for cfg in configs:
        if cfg["family"] == 1:
            assert bulk_plan(cfg, 5631, 2047, True) is None
            assert bulk_plan(cfg, 64, 64, True, w_aligned=False) is None


@pytest.mark.parametrize("shape", CORRECTNESS + EXTRA + [(4096, 1792), (4096, 2752), (4096, 1376)])
def test_rbulk_plan_and_coverage(configs, shape):
    h, i = shape
    ran = 0
    for cfg in configs:
        if cfg["family"] != 2:
            continue
        for rows, cols, gated in ((i, h, True), (h, i, False)):
            ran += audit_rbulk(cfg, rows, cols, gated)
    if h % 8 == 0 and i % 8 == 0 and max(h, i) <= 8192:
        assert ran > 0


def test_rbulk_covers_the_layer_shapes(configs):
    """Some RBULK geometry runs every gate and down shape of the benchmarked layers (and TP shards)."""
    for rows, cols, gated in ((14336, 4096, True), (4096, 14336, False), (11008, 4096, True),
                              (4096, 11008, False), (5632, 2048, True), (2048, 5632, False),
                              (1792, 4096, True), (4096, 1792, False), (7168, 4096, True), (4096, 7168, False)):
        plans = [rbulk_plan(c, rows, cols, gated) for c in configs if c["family"] == 2]
        assert any(p is not None for p in plans), (rows, cols)


def sbulk_layout(nm, rs, cols, stages, cw):
    def up(v, a):
        return (v + a - 1) // a * a
    full = up(stages * rs * nm * cols * 2, 16)
    empty = full + stages * 8
    meta = empty + stages * 8
    cnt = meta + stages * 8
    part = up(cnt + stages * 4, 16)
    return {"full": full, "empty": empty, "meta": meta, "cnt": cnt, "part": part,
            "total": up(part + stages * rs * cw * nm * 4, 16)}


def sbulk_plan(cfg, rows, cols, gated, w_aligned=True):
    """Mirror of launch_sbulk: None when the fallback geometry runs."""
    nm = 2 if gated else 1
    cw, cps, maxj, target, smax = cfg["warps"], cfg["rows"], cfg["unroll"], cfg["chunk"], cfg["stages"]
    nv = cols // 8
    ok = cols % 8 == 0 and w_aligned and nv <= maxj * cw * 32
    resident = SMS * cps
    budget = min(SMEM_PER_CTA, SMEM_PER_SM // cps - 1024) - 128
    rs = max(1, target // max(nm * cols * 2, 1))
    stages = 0
    while rs >= 1:
        stages = smax
        while stages >= 2 and sbulk_layout(nm, rs, cols, stages, cw)["total"] > budget:
            stages -= 1
        if stages >= 2 or rs == 1:
            break
        rs = rs // 2 if rs > 1 else 0
    if not ok or rs < 1 or stages < 2:
        return None
    per = (rows + resident * 16 - 1) // (resident * 16)
    rpb = max(rs, (per + rs - 1) // rs * rs)
    blocks = (rows + rpb - 1) // rpb
    stride = max(1, blocks // resident)
    while math.gcd(stride, blocks) != 1:
        stride += 1
    return {"rs": rs, "stages": stages, "rpb": rpb, "blocks": blocks, "stride": stride, "budget": budget,
            "layout": sbulk_layout(nm, rs, cols, stages, cw)}


def audit_sbulk(cfg, rows, cols, gated):
    plan = sbulk_plan(cfg, rows, cols, gated)
    if plan is None:
        return False
    nm = 2 if gated else 1
    rs, rpb, L = plan["rs"], plan["rpb"], plan["layout"]
    assert L["total"] <= plan["budget"] and L["full"] % 16 == 0 and L["part"] % 16 == 0
    assert L["meta"] % 8 == 0 and rpb % rs == 0
    owner = np.zeros(rows, np.int64)
    seen = set()
    for block in range(plan["blocks"]):  # every CTA index is one block, run by its CTA or its thief
        rb = block * plan["stride"] % plan["blocks"]
        seen.add(rb)
        b0, b1 = rb * rpb, min(rb * rpb + rpb, rows)
        assert b0 < rows
        for row in range(b0, b1, rs):
            ru = min(rs, b1 - row)
            nbytes = ru * cols * 2
            assert nbytes % 16 == 0 and (2 * row * cols) % 16 == 0 and nbytes * nm < (1 << 20)
            owner[row:row + ru] += 1
    assert (owner == 1).all() and len(seen) == plan["blocks"]
    return True


@pytest.mark.parametrize("shape", CORRECTNESS + EXTRA + [(4096, 1792), (4096, 2752), (4096, 1376)])
def test_sbulk_plan_and_coverage(configs, shape):
    h, i = shape
    ran = 0
    for cfg in configs:
        if cfg["family"] != 3:
            continue
        for rows, cols, gated in ((i, h, True), (h, i, False)):
            ran += audit_sbulk(cfg, rows, cols, gated)
    if h % 8 == 0 and i % 8 == 0 and max(h, i) <= 8192:
        assert ran > 0


def test_sbulk_blocks_leave_work_to_steal(configs):
    """At the layer shapes every resident CTA starts with many blocks left in the grid."""
    for cfg in configs:
        if cfg["family"] != 3:
            continue
        for rows, cols, gated in ((14336, 4096, True), (4096, 14336, False)):
            plan = sbulk_plan(cfg, rows, cols, gated)
            if plan is not None:
                assert plan["blocks"] >= 4 * SMS * cfg["rows"], (cfg["id"], plan)


LAYER_GEOMS = {200: (8, 1, 32768, 8), 203: (16, 1, 32768, 8), 201: (4, 2, 32768, 4), 202: (8, 2, 16384, 8),
               204: (4, 2, 16384, 8), 205: (8, 1, 16384, 12)}


def layer_plan(cfg_id, hidden, inter):
    """Mirror of launch_layer (csrc/swiglu_b200.cu)."""
    cw, cps, target, smax = LAYER_GEOMS[cfg_id]
    ct = cw * 32
    if hidden % 8 or inter % 8 or hidden // 8 > 8 * ct or inter // 8 > 8 * ct:
        return None
    G = min(SMS * cps, inter, hidden)
    row1, row2 = 4 * hidden, 2 * inter
    stage = -(-max(target, row1, row2) // 16) * 16
    rpc1, rpc2 = -(-inter // G), -(-hidden // G)
    budget = min(SMEM_PER_CTA, SMEM_PER_SM // cps - 1024) - 128

    def total(stages):
        up = lambda v, a: -(-v // a) * a  # noqa: E731
        full = up(stages * stage, 16)
        part1 = up(full + 16 * stages, 16)
        part2 = up(part1 + rpc1 * cw * 8, 16)
        return up(part2 + rpc2 * cw * 4, 16)
    stages = smax
    while stages >= 2 and total(stages) > budget:
        stages -= 1
    if stages < 2:
        return None
    return {"G": G, "stage": stage, "stages": stages, "rs1": max(1, min(stage // row1, rpc1)),
            "rs2": max(1, min(stage // row2, rpc2)), "total": total(stages), "budget": budget}


def test_layer_kernel_plans_cover_both_phases():
    assert layer_plan(200, 2047, 5631) is None
    for hidden, inter in ((4096, 14336), (4096, 11008), (2048, 8192), (2048, 5632), (512, 1376), (64, 96),
                          (4096, 7168), (4096, 3584), (4096, 1792), (1024, 256)):
        plans = {c: layer_plan(c, hidden, inter) for c in LAYER_GEOMS}
        assert plans[200] is not None or plans[203] is not None, (hidden, inter)
        for c, plan in plans.items():
            if plan is None:
                continue
            assert plan["total"] <= plan["budget"] and plan["G"] <= 1024
            assert plan["rs1"] * 4 * hidden <= plan["stage"] and plan["rs2"] * 2 * inter <= plan["stage"]
            for rows, cols, rs, nm in ((inter, hidden, plan["rs1"], 2), (hidden, inter, plan["rs2"], 1)):
                owner = np.zeros(rows, np.int64)
                for b in range(plan["G"]):
                    r0, r1 = b * rows // plan["G"], (b + 1) * rows // plan["G"]
                    assert r1 > r0
                    for row in range(r0, r1, rs):
                        ru = min(rs, r1 - row)
                        assert (ru * cols * 2) % 16 == 0 and (row * cols * 2) % 16 == 0
                        assert nm * ru * cols * 2 < (1 << 20)
                        owner[row:row + ru] += 1
                assert (owner == 1).all()


# ------------------------------------------- streaming whole layer (ids 220+)

STREAM_GEOMS = {220: (8, 2, 2, 8, 32768, 4), 221: (8, 1, 2, 16, 32768, 6), 223: (4, 2, 1, 16, 32768, 4)}
STREAM_MAX_BLOCKS = 8192 // 4 - 64


def stream_plan(cfg_id, hidden, inter):
    """Mirror of launch_stream_layer (csrc/swiglu_b200.cu): None where the kernel refuses."""
    cw, cps, rsplit, maxr, target, smax = STREAM_GEOMS[cfg_id]
    ct = cw * 32
    cb = 8 * ct // rsplit
    if hidden % 8 or inter % 8 or hidden // 8 > 8 * ct:
        return None
    G = min(SMS * cps, inter, hidden)
    rpc1, rpc2 = -(-inter // G), -(-hidden // G)
    if -(-rpc2 // rsplit) > maxr or -(-inter // cb) > STREAM_MAX_BLOCKS:
        return None
    rs1 = max(1, min(max(1, target // (4 * hidden)), 1 + (cb - 1) // G, rpc1))
    up = lambda v, a: -(-v // a) * a  # noqa: E731
    stage = up(max(rs1 * 4 * hidden, rpc2 * cb * 2), 16)
    budget = min(SMEM_PER_CTA, SMEM_PER_SM // cps - 1024) - 128

    units1 = -(-rpc1 // rs1)
    nblk = -(-inter // cb)
    if inter > 16384:  # h is held whole in shared memory
        return None

    def layout(stages):
        full = up(stages * stage, 16)
        gdone = full + 16 * stages           # full, empty barriers; then one per gate stage
        hready = gdone + 8 * units1          # one per block of h
        hsm = up(hready + 8 * nblk, 16)      # the CTA's fp16 copy of h
        bias = up(hsm + inter * 2, 16)
        part1 = up(bias + rpc1 * 8, 16)
        part2 = up(part1 + rpc1 * cw * 8, 16)
        return {"gdone": gdone, "hsm": hsm, "bias": bias, "part1": part1, "part2": part2,
                "total": up(part2 + rpc2 * cw * 4, 16)}
    stages = smax
    while stages >= 2 and layout(stages)["total"] > budget:
        stages -= 1
    if stages < 2:
        return None
    return {"G": G, "cw": cw, "ct": ct, "rsplit": rsplit, "maxr": maxr, "cb": cb, "rs1": rs1, "stage": stage,
            "stages": stages, "rpc1": rpc1, "rpc2": rpc2, "units1": units1, "budget": budget,
            "layout": layout(stages)}


@pytest.mark.parametrize("hidden,inter", [(4096, 14336), (4096, 11008), (2048, 8192), (2048, 5632), (512, 1376),
                                          (64, 96), (4096, 7168), (4096, 3584), (4096, 1792), (4096, 2752),
                                          (4096, 1376), (1024, 256), (520, 1032)])
def test_stream_layer_plans_and_coverage(hidden, inter):
    """Every copy of stream_layer_kernel stays in its stage and in its matrix, 16-byte aligned;
    every gate row and every Wd element is streamed once; the block words, shared arrays and
    row slots are indexed within their sizes; a stage's gate rows touch at most two h blocks."""
    plans = {c: stream_plan(c, hidden, inter) for c in STREAM_GEOMS}
    assert any(p is not None for p in plans.values()), (hidden, inter)
    for c, p in plans.items():
        if p is None:
            continue
        G, cb, rs1, stage, cw = p["G"], p["cb"], p["rs1"], p["stage"], p["cw"]
        assert p["layout"]["total"] <= p["budget"] and G <= 1024
        nblk = -(-inter // cb)
        gate_owner = np.zeros(inter, np.int64)
        wd_owner = np.zeros((hidden, nblk), np.int64)
        blk_rows = np.zeros(nblk, np.int64)
        for b in range(G):
            nA = (inter - b + G - 1) // G if b < inter else 0
            assert nA <= p["rpc1"] and -(-nA // rs1) <= p["units1"]  # one gate-stage barrier each
            for k in range(0, nA, rs1):  # one gate stage
                ru = min(rs1, nA - k)
                rows = [b + (k + i) * G for i in range(ru)]
                assert all(r < inter for r in rows)
                assert len({r // cb for r in rows}) <= 2 and rows[-1] // cb - rows[0] // cb <= 1
                for i, r in enumerate(rows):
                    for dst in (i * hidden * 2, (rs1 + i) * hidden * 2):
                        assert dst % 16 == 0 and dst + hidden * 2 <= stage
                    assert (r * hidden * 2) % 16 == 0 and (hidden * 2) % 16 == 0
                    gate_owner[r] += 1
                    blk_rows[r // cb] += 1
                assert (k + ru - 1) * cw * 2 + 2 * cw <= p["rpc1"] * cw * 2  # part1 slots
            d0, d1 = b * hidden // G, (b + 1) * hidden // G
            nD = d1 - d0
            assert 1 <= nD <= p["rpc2"] <= p["rsplit"] * p["maxr"]
            for cc in range(nblk):  # one down stage
                c0 = cc * cb
                seg = min(cb, inter - c0)
                assert seg % 8 == 0
                for r in range(nD):
                    dst = r * cb * 2
                    assert dst % 16 == 0 and dst + seg * 2 <= stage
                    assert ((d0 + r) * inter * 2 + c0 * 2) % 16 == 0 and (seg * 2) % 16 == 0
                    wd_owner[d0 + r, cc] += 1
        assert (gate_owner == 1).all() and (wd_owner == 1).all()
        # the block words count exactly the rows each block holds; the loader's 16-byte copies of
        # a block stay inside the shared copy of h
        assert all(blk_rows[cc] == min(cb, inter - cc * cb) for cc in range(nblk))
        for cc in range(nblk):
            c0, seg = cc * cb, min(cb, inter - cc * cb)
            assert (c0 * 2) % 16 == 0 and c0 + (seg // 8) * 8 <= inter and seg % 8 == 0
        # phase-2 thread map: slot t // VPB, vector t % VPB; rows slot + RSPLIT i cover [0, rpc2) once
        vpb = p["ct"] // p["rsplit"]
        assert vpb % 32 == 0 and vpb * 8 == cb
        cover = np.zeros(p["rpc2"], np.int64)
        for slot in range(p["rsplit"]):
            for i in range(p["maxr"]):
                r = slot + p["rsplit"] * i
                if r < p["rpc2"]:
                    cover[r] += 1
                    assert r * cw + (vpb - 1) // 32 < p["rpc2"] * cw  # part2 slot
        assert (cover == 1).all()


# ------------------------------------------------- grouped rows (stage_rows)

def reduce_scatter(values, K):
    """warp_reduce_scatter<K> (csrc/kernels.cuh) on 32 lanes x K float32 values: lane -> total."""
    v = [[np.float32(x) for x in values[lane]] for lane in range(32)]
    k, d = K, 16
    while k > 1:
        nxt = []
        for lane in range(32):
            p = lane ^ d
            upper, p_upper = bool(lane & d), bool(p & d)
            row = list(v[lane])
            for i in range(k // 2):
                keep = v[lane][i + k // 2] if upper else v[lane][i]
                recv = v[p][i] if p_upper else v[p][i + k // 2]  # what the partner sends
                row[i] = np.float32(keep + recv)
            nxt.append(row)
        v, k, d = nxt, k // 2, d // 2
    lk = int(math.log2(K))
    t = [v[lane][0] for lane in range(32)]
    d = 16 >> lk
    while d:
        t = [np.float32(t[lane] + t[lane ^ d]) for lane in range(32)]
        d //= 2
    return t


@pytest.mark.parametrize("nm", [1, 2])
@pytest.mark.parametrize("rg", [1, 2, 4, 8])
def test_stage_rows_group_reduction_and_writers(rg, nm):
    """Each row of a group is summed over all 32 lanes and stored exactly once, by the lane
    holding it (lane & (32/K - 1) == 0, value index lane >> (5 - log2 K)), and rows past the
    stage's end are not stored."""
    K = rg * nm
    if K > 8:
        pytest.skip("not instantiated")
    rng = np.random.default_rng(K)
    vals = rng.standard_normal((32, K)).astype(np.float32)
    totals = reduce_scatter(vals, K)
    lk = int(math.log2(K))
    for ru in range(1, rg + 1):  # rows present in the group
        written = {}
        for lane in range(32):
            if lane & ((32 >> lk) - 1):
                continue
            idx = lane >> (5 - lk)
            g, m = idx // nm, idx % nm
            if g < ru:
                assert (g, m) not in written
                written[(g, m)] = totals[lane]
        assert set(written) == {(g, m) for g in range(ru) for m in range(nm)}
        for (g, m), t in written.items():
            assert abs(t - vals[:, g * nm + m].astype(np.float64).sum()) < 1e-4


# ----------------------------------------------- tensor-parallel exchange slots

@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("hidden,cps", [(4096, 2), (4096, 1), (2048, 2), (520, 2)])
def test_exchange_slot_map(world, hidden, cps):
    """tp_exchange_rows (csrc/kernels.cuh): every store lands inside the receiving rank's
    2 x world x rows slots; in one call each slot a reader waits on is written by exactly one
    CTA of exactly one peer (the same CTA index: every rank runs the same grid), never twice;
    a rank never reads its own slot (it keeps its partial in registers); and the two
    parities of consecutive calls never share a slot."""
    G = min(SMS * cps, hidden)
    n_slots = 2 * world * hidden
    for epoch in (1, 2):
        par = epoch & 1
        writes = np.zeros((world, n_slots), np.int64)   # [receiving rank][slot]
        writer_cta = -np.ones((world, n_slots), np.int64)
        for src in range(world):
            for b in range(G):
                r0, r1 = b * hidden // G, (b + 1) * hidden // G
                for q in range(world):
                    if q == src:
                        continue
                    idx = (par * world + src) * hidden + np.arange(r0, r1)
                    assert idx.min(initial=0) >= 0 and idx.max(initial=0) < n_slots
                    writes[q, idx] += 1
                    writer_cta[q, idx] = b
        for me in range(world):
            for b in range(G):
                r0, r1 = b * hidden // G, (b + 1) * hidden // G
                for q in range(world):
                    if q == me:
                        continue
                    idx = par * world * hidden + q * hidden + np.arange(r0, r1)  # mine + q*rows + r0 + i
                    assert (writes[me, idx] == 1).all() and (writer_cta[me, idx] == b).all()
            own = par * world * hidden + me * hidden + np.arange(hidden)
            assert (writes[me, own] == 0).all()
        assert writes.max(initial=0) <= 1
        other = (1 - par) * world * hidden + np.arange(world * hidden)
        assert (writes[:, other] == 0).all()
