"""C ABI surface and the host-side planner. CPU only: nothing here launches a
kernel (the library loads without a GPU; the planner is pure host code)."""
import re

import numpy as np
import pytest

from conftest import REPO


@pytest.fixture(scope="module")
def lib():
    from d2sd_b200 import build
    build.build()
    from d2sd_b200 import _lib
    return _lib.load()


def header_prototypes():
    text = (REPO / "include" / "d2sd.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    protos = {}
    for m in re.finditer(r"^\s*[\w\s\*]+?\b(d2sd_\w+)\s*\(([^)]*)\)\s*;", text, flags=re.M):
        args = m.group(2).strip()
        n = 0 if args in ("", "void") else args.count(",") + 1
        protos[m.group(1)] = n
    return protos


def test_header_declares_the_entry_points():
    protos = header_prototypes()
    for name in ("d2sd_prefix_plan", "d2sd_prefix_attention", "d2sd_suffix_merge",
                 "d2sd_merge_state", "d2sd_verify_accept", "d2sd_commit_kv"):
        assert name in protos


def test_library_exports_every_declared_symbol(lib):
    from d2sd_b200 import _lib
    for name, nargs in header_prototypes().items():
        fn = getattr(lib, name)  # raises if not exported
        assert fn is not None
        assert name in _lib.SIGNATURES, name
        assert len(_lib.SIGNATURES[name][1]) == nargs, name
    assert lib.d2sd_version() >= 100


def test_invalid_arguments_raise(lib):
    from d2sd_b200 import ops
    with pytest.raises(ValueError):
        ops.prefix_plan([4], [0], [5], [3], 32, 8, 148)  # kv_end < kv_start
    with pytest.raises(ValueError):
        ops.prefix_plan([4], [0], [0], [3], 30, 8, 148)  # heads not a multiple
    with pytest.raises(NotImplementedError):
        ops.prefix_plan([4], [0], [0], [3], 24, 8, 148)  # G = 3 does not divide 128
    assert lib.d2sd_verify_accept(None, 1, 1, 1, 1, 0, 0, None, 0, 0, None, None, None, None,
                                  0, None) == 1
    assert "invalid" in lib.d2sd_last_error().decode()


def decode(plan):
    H = dict(num_ctas=plan[1], num_items=plan[2], num_units=plan[3], num_req=plan[4],
             num_slots=plan[5], num_tok=plan[6], off_cta=plan[7], off_items=plan[8],
             off_units=plan[9], off_req=plan[10], off_tok=plan[11], G=plan[12], Hk=plan[13],
             gs=plan[14])
    cta = plan[H["off_cta"]:H["off_cta"] + H["num_ctas"] + 1]
    items = plan[H["off_items"]:H["off_items"] + 12 * H["num_items"]].reshape(-1, 12)
    units = plan[H["off_units"]:H["off_units"] + 2 * H["num_units"]].reshape(-1, 2)
    reqs = plan[H["off_req"]:H["off_req"] + 4 * H["num_req"]].reshape(-1, 4)
    toks = plan[H["off_tok"]:H["off_tok"] + H["num_tok"]]
    return H, cta, items, units, reqs, toks


@pytest.mark.parametrize("case", [
    dict(q=[256], kv=[(0, 32768)], Hq=32, Hk=8, sms=148),          # north star (k = 0)
    dict(q=[200], kv=[(0, 32768)], Hq=32, Hk=8, sms=148),          # tree, k = 8
    dict(q=[64] * 64, kv=[(0, int(L)) for L in np.random.default_rng(0).integers(512, 8193, 64)],
         Hq=32, Hk=8, sms=148),                                     # batched serving
    dict(q=[96], kv=[(16384 - 128, 16384)], Hq=64, Hk=8, sms=148),   # GPT-OSS sliding layer
    dict(q=[96], kv=[(0, 16384)], Hq=64, Hk=8, sms=148),            # GPT-OSS full layer
    # one rank's share under KV-head sharding: north star on 2, 4 and 8 GPUs,
    # GPT-OSS full layer on 8
    dict(q=[256], kv=[(0, 32768)], Hq=16, Hk=4, sms=148),
    dict(q=[256], kv=[(0, 32768)], Hq=8, Hk=2, sms=148),
    dict(q=[256], kv=[(0, 32768)], Hq=4, Hk=1, sms=148),
    dict(q=[96], kv=[(0, 16384)], Hq=8, Hk=1, sms=148),
    dict(q=[64, 3, 0, 17], kv=[(0, 5), (0, 0), (0, 100), (7, 300)], Hq=8, Hk=2, sms=10),
    dict(q=[64], kv=[(0, 512)], Hq=32, Hk=8, sms=1),
])
def test_plan_covers_every_column_once(lib, case):
    from d2sd_b200 import ops
    R = len(case["q"])
    offs = np.concatenate([[0], np.cumsum(case["q"])[:-1]]).astype(int).tolist()
    ks = [a for a, _ in case["kv"]]
    ke = [b for _, b in case["kv"]]
    plan, nslots = ops.prefix_plan(case["q"], offs, ks, ke, case["Hq"], case["Hk"], case["sms"])
    H, cta, items, units, reqs, toks = decode(plan)
    G = case["Hq"] // case["Hk"]
    assert H["G"] == G and H["num_slots"] == nslots
    assert H["num_ctas"] <= case["sms"]
    assert np.all(np.diff(cta) >= 0) and cta[-1] == H["num_items"]
    # coverage: every (request, head, query tile, kv tile) exactly once
    seen = {}
    slot_owner = {}
    for it in items:
        r, h, qt0, has1, t0, t1, s0, e0, sl0, sl1, qtok = it[:11]
        assert t1 > t0
        for qt, sl in ((qt0, sl0), (qt0 + 1, sl1)):
            if qt == qt0 + 1 and not has1:
                assert sl == -1
                continue
            assert 0 <= sl < nslots and sl not in slot_owner
            slot_owner[sl] = (r, h, qt)
            for t in range(t0, t1):
                key = (r, h, qt, t)
                assert key not in seen
                seen[key] = True
        assert qtok == offs[r] + qt0 * (128 // G)
    expected = set()
    for r in range(R):
        nqt = -(-case["q"][r] * G // 128)
        s, e = ks[r], ke[r]
        if e <= s or case["q"][r] == 0:
            continue
        for h in range(case["Hk"]):
            for qt in range(nqt):
                for t in range(s // 128, -(-e // 128)):
                    expected.add((r, h, qt, t))
    assert set(seen) == expected
    # units: contiguous slot ranges owned by exactly that unit
    for r in range(R):
        ub, nqt, qo, qn = reqs[r]
        assert qo == offs[r] and qn == case["q"][r]
        for h in range(case["Hk"]):
            for qt in range(nqt):
                base, n = units[ub + h * nqt + qt]
                for s in range(base, base + n):
                    assert slot_owner[s] == (r, h, qt)
        for t in range(case["q"][r]):
            assert toks[offs[r] + t] == r
    # balance: no CTA gets much more than its share of columns
    work = np.zeros(H["num_ctas"])
    for c in range(H["num_ctas"]):
        for it in items[cta[c]:cta[c + 1]]:
            work[c] += it[5] - it[4]
    if H["num_ctas"] > 1 and work.sum() > 10 * H["num_ctas"]:
        assert work.max() <= work.mean() * 1.15 + 2


def test_plan_groups_share_kv_stream(lib):
    """North-star shape: the 4 query-tile pairs of a kv head walk the same KV
    tiles in the 4 adjacent CTAs of a group."""
    from d2sd_b200 import ops
    plan, _ = ops.prefix_plan([256], [0], [0], [32768], 32, 8, 148)
    H, cta, items, *_ = decode(plan)
    assert H["gs"] == 4 and H["num_ctas"] == 148
    for g in range(H["num_ctas"] // 4):
        lists = [items[cta[4 * g + k]:cta[4 * g + k + 1]] for k in range(4)]
        for k in range(1, 4):
            assert np.array_equal(lists[k][:, [0, 1, 4, 5]], lists[0][:, [0, 1, 4, 5]])
            assert np.all(lists[k][:, 2] == lists[0][:, 2] + 2 * k)


def test_truncation_bias_constant():
    """The mean relative loss of truncating f32 softmax weights to bf16 (the
    constant kernel (a) divides out of O) for weights spread over many octaves:
    half a last place, 2^-8 / m for mantissa m, averaged over log-uniform m,
    2^-8 / (2 ln 2) = 0.2818%."""
    import re
    from pathlib import Path
    src = (Path(__file__).resolve().parents[1] / "d2sd_b200" / "csrc" / "prefix_attn.cu").read_text()
    c = float(re.search(r"kTruncBias = 1\.0f / \(1\.0f - ([0-9.]+)f\)", src).group(1))
    rng = np.random.default_rng(0)
    p = np.exp2(rng.uniform(-20.0, 8.0, 2_000_000)).astype(np.float32)
    tr = (p.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)
    loss = 1.0 - float(np.mean(tr / p))
    assert abs(loss - c) < 2e-5, (loss, c)
    assert abs(c - 2.0 ** -8 / (2.0 * np.log(2.0))) < 1e-5
