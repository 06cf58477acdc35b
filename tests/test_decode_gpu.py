"""End-to-end decode parity on the GPU: the Engine (GGUF load -> C-ABI kernels ->
recorded token plan, or the fused token kernel) against the CPU oracle on the
same synthetic GGUF.

Checks, per token: every layer's hidden state (relative error <= 1e-2, the
north-star bound), the final logits, and the greedy ids over the decode window.

Why not ~1e-6: activations are stored in f16 where the reference stores f16,
and on these random-weight models a perturbation of 1e-6 (relative) before the
f16 roundings already moves a layer's hidden state by ~2e-4 (measured on the
oracle itself), so two correct implementations whose f32 sums differ only in
order agree to ~1e-3..1e-2 after a few layers.  A greedy id may therefore only
differ where the oracle's top-2 logit margin is below TIE (5e-3 absolute; the
logits have a standard deviation of ~0.45) -- a tie within that noise.
"""
import numpy as np
import pytest

from oracle.model import OracleModel

pytestmark = pytest.mark.gpu
HIDDEN_TOL = 1e-2
TIE = 5e-3


def _rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


PATHS = [("tiny", False), ("tiny", True), ("tiny_ple", False), ("tiny_ple", True), ("tiny_moe", False)]


@pytest.mark.parametrize("name,fused", PATHS)
def test_teacher_forced_layers(e4b, models, name, fused):
    """Step both models through the same tokens; compare every layer, every step
    (fused: the whole token as one persistent kernel; else one kernel per operator)."""
    buf = models(name)
    eng = e4b.Engine(buf, 0, record=True, fused=fused)
    ref = OracleModel(buf)
    toks = e4b.synth.prompt_ids(40, eng.cfg.vocab, seed=3)     # > ring of the sliding layers (24)
    worst = 0.0
    try:
        for pos, t in enumerate(toks):
            eng.step(int(t), pos)
            eng.dev.sync()
            rid, rec = ref.step(int(t), pos, record=True)
            dump = eng.read_dump()
            for l in range(eng.cfg.layers):
                worst = max(worst, _rel(dump[l], rec["hidden"][l]))
            lg = eng.read_logits()
            assert _rel(lg, rec["logits"]) < HIDDEN_TOL
            top2 = np.sort(rec["logits"])[-2:]
            if eng.argmax_fast() != rid:
                assert top2[1] - top2[0] < TIE, (pos, eng.argmax_fast(), rid)
        assert eng.dev.status() == 0
    finally:
        eng.close()
    assert worst < HIDDEN_TOL, worst
    print(f"{name}: worst per-layer hidden rel err {worst:.2e}")


@pytest.mark.parametrize("name,P,N,fused", [("tiny", 32, 32, False), ("tiny", 32, 32, True),
                                            ("tiny_ple", 20, 24, False), ("tiny_ple", 20, 24, True),
                                            ("tiny_moe", 16, 24, False)])
def test_greedy_ids_match(e4b, models, name, P, N, fused):
    """benchmark config 1 shape for tiny: 32-token prompt (seed 0), 32 greedy tokens."""
    buf = models(name)
    prompt = e4b.synth.prompt_ids(P, e4b.config.get(name).vocab, seed=0)
    eng = e4b.Engine(buf, 0, fused=fused)
    try:
        ids = eng.generate(prompt, N)
        again = eng.generate(prompt, N)          # rerun on the same engine: caches need no reset
    finally:
        eng.close()
    rids, margins, _ = OracleModel(buf).generate(prompt, N, record=True)
    assert ids == again
    for i, (a, b) in enumerate(zip(ids, rids)):
        if a != b:
            assert margins[i] < TIE, (i, a, b, margins[i])
            break


def test_fused_matches_operator_path(e4b, models):
    """The fused token kernel and the per-operator kernels agree on the same
    tokens within the parity bound (both f32 with f16 activations; summation
    orders differ, which the f16 roundings amplify to ~1e-3, see above)."""
    buf = models("tiny_ple")
    a = e4b.Engine(buf, 0, record=True, fused=True)
    b = e4b.Engine(buf, 0, record=True, fused=False)
    worst = 0.0
    try:
        for pos, t in enumerate(e4b.synth.prompt_ids(30, a.cfg.vocab, seed=5)):
            a.step(int(t), pos)
            b.step(int(t), pos)
            a.dev.sync()
            b.dev.sync()
            worst = max(worst, _rel(a.read_dump(), b.read_dump()))
        assert a.dev.status() == 0 and b.dev.status() == 0
    finally:
        a.close()
        b.close()
    assert worst < HIDDEN_TOL, worst
    print(f"fused vs per-operator: worst per-layer hidden rel diff {worst:.2e}")


def test_fused_deterministic(e4b, models):
    """Fixed partition and merge order: two runs give bit-identical states."""
    buf = models("tiny_ple")
    outs = []
    for _ in range(2):
        eng = e4b.Engine(buf, 0, record=True, fused=True)
        try:
            for pos, t in enumerate(e4b.synth.prompt_ids(12, eng.cfg.vocab, seed=9)):
                eng.step(int(t), pos)
            eng.dev.sync()
            outs.append((eng.read_dump().copy(), eng.read_logits().copy()))
        finally:
            eng.close()
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])


def _sync_caches(eng, ref):
    """Give the engine the oracle's KV caches (identical f16 layout), so one
    step is compared from identical state."""
    for L in eng.layers:
        eng.dev.write(L.kc, np.ascontiguousarray(ref.kc[L.i]), 0)
        eng.dev.write(L.vc, np.ascontiguousarray(ref.vc[L.i]), 0)


def _perturbed_step(ref, pert, tok, pos, seed):
    """One oracle step from `ref`'s caches with every f16 rounding input scaled by
    (1 + 1e-6 N(0,1)): the oracle's own sensitivity to f32 summation order."""
    from oracle import ops as O
    for l in range(ref.L):
        pert.kc[l][...] = ref.kc[l]
        pert.vc[l][...] = ref.vc[l]
    pert.kv_count = ref.kv_count
    rng = np.random.default_rng(seed)
    orig = O.f16r

    def noisy(x):
        x = np.asarray(x, np.float32)
        return orig((x * (1 + 1e-6 * rng.standard_normal(x.shape))).astype(np.float32))
    O.f16r = noisy
    try:
        return pert.step(int(tok), pos, record=True)[1]
    finally:
        O.f16r = orig


def test_e4b_fused_matches_oracle(e4b):
    """Full E4B shapes (35 layers, FF 16384, PLE, sliding + global layers): the
    fused kernel against the oracle, every layer, every step, each step from the
    oracle's KV caches (so errors do not compound across positions).

    Bound: 1e-2 relative, or -- at positions where this random-weight model is
    so sensitive that the oracle itself moves further under a 1e-6 perturbation
    before its f16 roundings -- 3x what that perturbation produces (attention
    over near-tied keys turns tiny score differences into ~1e-2 output changes)."""
    buf = e4b.synth.build_model(e4b.config.e4b())
    eng = e4b.Engine(buf, 0, record=True)
    assert eng.fused
    ref, pert = OracleModel(buf), OracleModel(buf)
    worst, report = 0.0, []
    try:
        for pos, t in enumerate(e4b.synth.prompt_ids(6, eng.cfg.vocab, seed=1)):
            _sync_caches(eng, ref)
            prec = _perturbed_step(ref, pert, t, pos, seed=100 + pos)
            eng.step(int(t), pos)
            eng.dev.sync()
            rid, rec = ref.step(int(t), pos, record=True)
            dump = eng.read_dump()
            err = max(_rel(dump[l], rec["hidden"][l]) for l in range(eng.cfg.layers))
            noise = max(_rel(prec["hidden"][l], rec["hidden"][l]) for l in range(eng.cfg.layers))
            lerr = _rel(eng.read_logits(), rec["logits"])
            lnoise = _rel(prec["logits"], rec["logits"])
            report.append((pos, err, noise, lerr, lnoise))
            assert err < max(HIDDEN_TOL, 3 * noise), report
            assert lerr < max(HIDDEN_TOL, 3 * lnoise), report
            worst = max(worst, err)
            if eng.argmax_fast() != rid:
                top2 = np.sort(rec["logits"])[-2:]
                assert top2[1] - top2[0] < TIE, (pos, eng.argmax_fast(), rid)
        assert eng.dev.status() == 0
        # free-running greedy decode from a fresh state: the first 4 ids agree
        # (further out, the growth of rounding differences described above makes
        # the top-2 logit gap the only meaningful criterion, tested per step above)
        prompt = e4b.synth.prompt_ids(6, eng.cfg.vocab, seed=2)
        for L in eng.layers:
            eng.dev.memset(L.kc, 0)
            eng.dev.memset(L.vc, 0)
        ids = eng.generate(prompt, 4)
    finally:
        eng.close()
    for r in report:
        print("pos %d: hidden err %.2e (oracle 1e-6 noise %.2e), logits err %.2e (noise %.2e)" % r)
    ref.reset()
    rids, margins, _ = ref.generate(prompt, 4, record=True)
    for i, (a, b) in enumerate(zip(ids, rids)):
        if a != b:
            assert margins[i] < TIE, (i, a, b, margins[i])
            break


def _window_check(got_ids, ref_ids, margins, dlog, max_flips=2):
    """Per-step greedy agreement over a window where both sides consumed the
    same tokens: a step may disagree only where the oracle's top-2 logit margin
    is a tie (< TIE) or is within twice that step's measured logit difference
    (the numerical error the step itself shows), and at most `max_flips` steps
    may disagree at all."""
    flips = [i for i, (a, b) in enumerate(zip(got_ids, ref_ids)) if a != b]
    for i in flips:
        assert margins[i] < max(TIE, 2 * dlog[i]), (i, got_ids[i], ref_ids[i], margins[i], dlog[i])
    assert len(flips) <= max_flips, flips


class _NoisyF16:
    """Within the block, every f16 rounding of the oracle first scales its input
    by (1 + 1e-6 N(0,1)): the oracle's own sensitivity to f32 summation order."""

    def __init__(self, seed):
        self.rng = np.random.default_rng(seed)

    def __enter__(self):
        from oracle import ops as O
        self.O, self.orig = O, O.f16r
        rng, orig = self.rng, self.orig

        def noisy(x):
            x = np.asarray(x, np.float32)
            return orig((x * (1 + 1e-6 * rng.standard_normal(x.shape))).astype(np.float32))
        O.f16r = noisy
        return self

    def __exit__(self, *a):
        self.O.f16r = self.orig


def test_e4b_greedy_window_64(e4b):
    """Full E4B shapes through the fused token kernel: a 16-token prompt then 64
    greedy steps, with the GPU engine, the oracle and a second oracle whose f16
    roundings see 1e-6 relative noise each on their own state, all fed the
    oracle's greedy token every step (so a disagreement does not end the
    comparison).  This 35-layer random-weight model amplifies rounding
    differences chaotically over positions (measured: logit differences of
    ~0.5 after 16 positions between the oracle and its own 1e-6 perturbation),
    so greedy identity over the window is not a property any two f32
    summation orders share.  Checked instead, per step: the GPU's logits are
    no further from the oracle than 3x the perturbed oracle's (or 1e-2 of the
    logit scale), every greedy disagreement lies within twice that step's
    measured logit difference, and the GPU disagrees with the oracle at most
    as often as the perturbed oracle does, plus 2."""
    buf = e4b.synth.build_model(e4b.config.e4b())
    eng = e4b.Engine(buf, 0)
    assert eng.fused
    ref, pert = OracleModel(buf), OracleModel(buf)
    prompt = [int(t) for t in e4b.synth.prompt_ids(16, eng.cfg.vocab, seed=3)]
    rows = []          # (step, gpu id, oracle id, perturbed id, margin, |dlog| gpu, |dlog| perturbed)
    try:
        tok = None
        for pos in range(len(prompt) + 64):
            t = prompt[pos] if pos < len(prompt) else tok
            eng.step(int(t), pos)
            rid, rec = ref.step(int(t), pos, record=True)
            with _NoisyF16(1000 + pos):
                pid, prec = pert.step(int(t), pos, record=True)
            if pos >= len(prompt) - 1:
                eng.dev.sync()
                lg = eng.read_logits()
                top2 = np.sort(rec["logits"])[-2:]
                rows.append((pos, int(np.argmax(lg)), rid, pid, float(top2[1] - top2[0]),
                             float(np.max(np.abs(lg - rec["logits"]))),
                             float(np.max(np.abs(prec["logits"] - rec["logits"])))))
            tok = rid
        assert eng.dev.status() == 0
    finally:
        eng.close()
    assert len(rows) == 65
    scale = 1e-2 * max(np.max(np.abs(rec["logits"])), 1.0)
    for r in rows:
        assert r[5] <= max(3 * r[6], scale), r
        if r[1] != r[2]:
            assert r[4] < max(TIE, 2 * r[5]), r
    flips_gpu = sum(r[1] != r[2] for r in rows)
    flips_pert = sum(r[3] != r[2] for r in rows)
    print(f"e4b window: {flips_gpu} GPU / {flips_pert} perturbed-oracle disagreements in {len(rows)} steps; "
          f"median |dlogits| {np.median([r[5] for r in rows]):.3f} GPU vs {np.median([r[6] for r in rows]):.3f}")
    assert flips_gpu <= flips_pert + 2, (flips_gpu, flips_pert)


def test_a4b_batch_engine_full_size(e4b):
    """Benchmark config 4 at full size (30 layers, hidden 2816, 128 experts top-8,
    vocabulary 262144) through the batched engine: two sequences, an 8-token
    prompt and 16 greedy steps each, both sides fed the oracle's greedy tokens;
    the greedy ids checked at every step of both sequences."""
    buf = e4b.synth.build_model(e4b.config.a4b())
    B, P, N = 2, 8, 16
    prompts = np.stack([e4b.synth.prompt_ids(P, 262144, seed=50 + b) for b in range(B)])
    eng = e4b.BatchEngine(buf, B, 0)
    refs = [OracleModel(buf) for _ in range(B)]
    got = [[] for _ in range(B)]
    want = [[] for _ in range(B)]
    margins = [[] for _ in range(B)]
    dlog = [[] for _ in range(B)]
    try:
        toks = prompts[:, 0].copy()
        for pos in range(P + N):
            if pos < P:
                toks = prompts[:, pos].copy()
            eng.step(toks, pos)
            nxt = np.empty(B, np.uint32)
            recs = []
            for b in range(B):
                rid, rec = refs[b].step(int(toks[b]), pos, record=True)
                nxt[b] = rid
                recs.append(rec)
            if pos >= P - 1:
                eng.dev.sync()
                lg = eng.read_logits()
                for b in range(B):
                    top2 = np.sort(recs[b]["logits"])[-2:]
                    got[b].append(int(np.argmax(lg[b])))
                    want[b].append(int(nxt[b]))
                    margins[b].append(float(top2[1] - top2[0]))
                    dlog[b].append(float(np.max(np.abs(lg[b] - recs[b]["logits"]))))
            toks = nxt
        assert eng.dev.status() == 0
    finally:
        eng.close()
    for b in range(B):
        _window_check(got[b], want[b], margins[b], dlog[b])
