"""Oracle (test infrastructure): sampling and speculative acceptance.

Two groups of functions:

1. Restatements of the reference (``androidllm/engine.py``):
   ``sample_reference`` (``engine.py:26-45``), its uniform-driven form
   ``sample_reference_u`` (numpy ``Generator.choice(n, p=p)`` is
   ``searchsorted(cumsum(float64 p) / cdf[-1], random(), 'right')``; checked
   against the reference by the golden tests), and ``accept_greedy``
   (``engine.py:306-320``: accept while the target's own pick equals the
   draft's candidate, then emit the target's correction or bonus token).

2. The min(1, p/q) rejection-sampling rule the product's GPU acceptance kernel
   implements.  The reference has no such rule (it accepts only when an
   independent target sample equals the draft sample), so this definition is
   pinned only against itself: parity unpinned by the reference.  Its
   arithmetic is fixed so a GPU can reproduce it bit for bit:

   * ``rexp``: exp from basic fp32 operations only (Cody-Waite range
     reduction ``x = k*ln2 + r`` and the degree-7 Taylor polynomial of e^r in
     Horner form, then an exact scaling by 2^k).  Each step is one correctly
     rounded IEEE fp32 operation, so numpy and CUDA (``__fmul_rn`` /
     ``__fadd_rn``, no contraction) give identical bits.
   * sums run in chunks of ``CHUNK`` elements: sequential inside a chunk,
     then sequential over chunk totals.
   * inverse-CDF sampling walks the same chunk totals, then the elements of
     the chosen chunk, and returns the first index whose running sum exceeds
     ``u * total``.
"""
import numpy as np

CHUNK = 256

# Cody-Waite split of ln(2): LN2_HI is fp32(ln2) with its low 9 mantissa bits
# cleared (0x3F317200), so k * LN2_HI is exact for |k| < 2**9; LN2_LO is
# fp32(ln2 - LN2_HI).  The CUDA side uses the same two bit patterns.
LOG2E = np.float32(1.4426950408889634)
LN2_HI = np.array([0x3F317200], dtype=np.uint32).view(np.float32)[0]
LN2_LO = np.float32(np.log(2.0) - float(LN2_HI))
_TAYLOR = [np.float32(1.0 / f) for f in (5040.0, 720.0, 120.0, 24.0, 6.0, 2.0, 1.0, 1.0)]
EXP_UNDERFLOW = np.float32(-87.0)


# --------------------------------------------------------------------------
# reference sampler (androidllm/engine.py:26-45)
# --------------------------------------------------------------------------

def _reference_probs(logits, temperature, top_p, min_p):
    """engine.py:27-43 up to the point where rng.choice is called.

    Returns ``(candidate_ids, probs)`` with probs the fp32 vector handed to
    ``rng.choice``.
    """
    lg = np.asarray(logits, dtype=np.float32).reshape(-1)
    p = np.exp((lg - np.max(lg)) / max(temperature, 1e-9))
    p = p / p.sum()
    if min_p and 0 < min_p < 1.0:
        keep = p >= min_p * p.max()
        if keep.any():
            p = np.where(keep, p, 0.0)
            p = p / p.sum()
    if top_p < 1.0:
        order = np.argsort(-p)
        cum = np.cumsum(p[order])
        ids = order[cum <= top_p]
        if len(ids) == 0:
            ids = order[:1]
        sub = p[ids] / p[ids].sum()
        return ids, sub
    return np.arange(p.size), p


def choice_u(p, u):
    """numpy ``Generator.choice(len(p), p=p)`` given its uniform draw ``u``."""
    cdf = np.asarray(p, dtype=np.float64).cumsum()
    cdf /= cdf[-1]
    return int(cdf.searchsorted(u, side="right"))


def sample_reference_u(logits, temperature, top_p, min_p, u):
    """engine.py:26-45 with the uniform drawn by ``rng.choice`` passed in."""
    if temperature <= 0:
        return int(np.argmax(np.asarray(logits, dtype=np.float32).reshape(-1)))
    ids, p = _reference_probs(logits, temperature, top_p, min_p)
    return int(ids[choice_u(p, u)])


def sample_reference(logits, temperature, top_p, min_p, rng):
    """engine.py:26-45 driven by a numpy Generator (consumes one draw if T > 0)."""
    if temperature <= 0:
        return int(np.argmax(np.asarray(logits, dtype=np.float32).reshape(-1)))
    ids, p = _reference_probs(logits, temperature, top_p, min_p)
    return int(ids[rng.choice(len(ids), p=p)])


def accept_greedy(target_tokens, draft_tokens):
    """engine.py:306-320: returns ``(emitted, n_accepted)``.

    ``target_tokens[i]`` is the target's pick after consuming the first ``i``
    candidates (``K + 1`` entries), ``draft_tokens`` the ``K`` candidates.
    """
    emitted = []
    for i, c in enumerate(draft_tokens):
        g = int(target_tokens[i])
        emitted.append(g)
        if g != int(c):
            return emitted, i
    emitted.append(int(target_tokens[len(draft_tokens)]))
    return emitted, len(draft_tokens)


# --------------------------------------------------------------------------
# reproducible probabilities and min(1, p/q) acceptance (builder-defined)
# --------------------------------------------------------------------------

def rexp(x):
    """exp(x) for fp32 ``x <= 0`` from correctly rounded fp32 operations only."""
    x = np.asarray(x, dtype=np.float32)
    k = np.rint(x * LOG2E).astype(np.float32)
    r = (x - k * LN2_HI) - k * LN2_LO
    acc = _TAYLOR[0]
    for c in _TAYLOR[1:]:
        acc = acc * r + c
    out = np.ldexp(acc, k.astype(np.int32)).astype(np.float32)
    return np.where(x < EXP_UNDERFLOW, np.float32(0.0), out).astype(np.float32)


def chunk_sums(v):
    """Sequential fp32 sum of each CHUNK-element chunk (last chunk may be short)."""
    v = np.asarray(v, dtype=np.float32)
    n = v.size
    pad = (-n) % CHUNK
    w = np.concatenate([v, np.zeros(pad, np.float32)]).reshape(-1, CHUNK)
    return np.cumsum(w, axis=1, dtype=np.float32)[:, -1]


def chunked_total(v):
    cs = chunk_sums(v)
    return np.cumsum(cs, dtype=np.float32)[-1]


def probs_repro(logits, temperature, min_p=0.0):
    """Sampling distribution softmax(l / T) (optionally min-p filtered), fp32.

    Same operations as engine.py:30-36 (``(l - max) / T``, exp, divide by the
    sum, min-p keep ``p >= min_p * max(p)``, renormalise) with ``rexp`` and the
    chunked summation order.
    """
    lg = np.asarray(logits, dtype=np.float32).reshape(-1)
    z = (lg - np.max(lg)) / np.float32(max(temperature, 1e-9))
    e = rexp(z)
    p = e / chunked_total(e)
    if min_p and 0 < min_p < 1.0:
        keep = p >= np.float32(min_p) * np.max(p)
        p = np.where(keep, p, np.float32(0.0)).astype(np.float32)
        p = p / chunked_total(p)
    return p.astype(np.float32)


def sample_probs(p, u):
    """Inverse CDF over ``p`` (fp32, non-negative) with the chunked order."""
    p = np.asarray(p, dtype=np.float32)
    cs = chunk_sums(p)
    total = np.cumsum(cs, dtype=np.float32)[-1]
    target = np.float32(u) * total
    acc = np.float32(0.0)
    for c in range(cs.size):
        nxt = np.float32(acc + cs[c])
        if nxt > target or c == cs.size - 1:
            lo = c * CHUNK
            hi = min(lo + CHUNK, p.size)
            last_pos = -1
            for j in range(lo, hi):
                if p[j] > 0:
                    last_pos = j
                acc = np.float32(acc + p[j])
                if acc > target and p[j] > 0:
                    return j
            return last_pos if last_pos >= 0 else int(np.flatnonzero(p > 0)[-1])
        acc = nxt
    raise AssertionError("unreachable")


def accept_rejection(p_target, q_draft, draft_tokens, u_accept, u_resample):
    """Speculative rejection sampling with the fixed arithmetic above.

    ``p_target``: (K+1, V) target distributions at the K+1 verify rows.
    ``q_draft``:  (K, V) draft distributions the candidates were drawn from.
    Candidate i is accepted iff ``u_accept[i] * q[i][x] < p[i][x]`` (one fp32
    product, i.e. ``u < min(1, p/q)`` for ``q > 0``).  At the first rejection
    the token is drawn from ``max(0, p_i - q_i)`` (normalised) with
    ``u_resample``; if every candidate is accepted the bonus token is drawn
    from ``p_K`` with the same ``u_resample``.  Returns ``(emitted, n_accepted)``.
    """
    p_target = np.asarray(p_target, dtype=np.float32)
    q_draft = np.asarray(q_draft, dtype=np.float32)
    emitted = []
    for i, x in enumerate(draft_tokens):
        x = int(x)
        if np.float32(np.float32(u_accept[i]) * q_draft[i, x]) < p_target[i, x]:
            emitted.append(x)
            continue
        resid = np.maximum(p_target[i] - q_draft[i], np.float32(0.0)).astype(np.float32)
        if not np.any(resid > 0):
            resid = p_target[i]
        emitted.append(sample_probs(resid, u_resample))
        return emitted, i
    emitted.append(sample_probs(p_target[len(draft_tokens)], u_resample))
    return emitted, len(draft_tokens)


# --------------------------------------------------------------------------
# the device sampler's arithmetic (engine.py:26-45 semantics, fixed order)
# --------------------------------------------------------------------------
# The GPU sampler follows engine.py:26-45 step for step (softmax of l / T,
# min-p keep and renormalise, top-p nucleus in descending-probability order,
# inverse CDF on one uniform draw) with this fixed arithmetic, restated here
# so tests can demand identical tokens:
#   * exp is ``rexp``;
#   * a row is split into SAMPLE_CTAS contiguous slices of ceil(V / SAMPLE_CTAS)
#     elements (one CTA of a thread-block cluster each); a sum is the
#     kernel's: in each slice thread t (of SAMPLE_THREADS) adds the slice's
#     elements t, t + SAMPLE_THREADS, ... in order, the 32 lanes of a warp are
#     added in lane order, the warp totals in warp order, and the slice
#     totals in slice order;
#   * probability masses are fixed point, floor(p * 2^52) as uint64, so the
#     nucleus and the CDF walk are exact integer arithmetic;
#   * the nucleus order is descending probability, ties by ascending index
#     (the reference's argsort leaves tie order to its sort implementation);
#   * temperature, top_p and min_p act as fp32 values, as numpy 2 applies a
#     Python float to fp32 arrays; the uniform draw is fp64.
# It differs from the reference only by fp32 rounding (its exp and pairwise
# sums), i.e. when a draw lands within rounding of a CDF or nucleus boundary.

SAMPLE_THREADS = 1024
SAMPLE_CTAS = 8
MASS_SCALE = float(2 ** 52)


def _slice_total(v):
    pad = (-v.size) % SAMPLE_THREADS
    w = np.concatenate([v, np.zeros(pad, np.float32)]).reshape(-1, SAMPLE_THREADS)
    per_thread = np.cumsum(w, axis=0, dtype=np.float32)[-1]
    per_warp = np.cumsum(per_thread.reshape(-1, 32), axis=1, dtype=np.float32)[:, -1]
    return np.cumsum(per_warp, dtype=np.float32)[-1]


def block_total(v):
    """The sampler's fixed-order fp32 sum of a row (see above)."""
    v = np.asarray(v, dtype=np.float32).reshape(-1)
    per = -(-v.size // SAMPLE_CTAS)
    acc = np.float32(0.0)
    for c in range(SAMPLE_CTAS):
        part = v[c * per:(c + 1) * per]
        if part.size:
            acc = np.float32(acc + _slice_total(part))
    return acc


def fixed_probs(logits, temperature, min_p=0.0):
    """engine.py:29-36 with the sampler's arithmetic: fp32 probabilities."""
    lg = np.asarray(logits, dtype=np.float32).reshape(-1)
    t = np.float32(max(float(temperature), 1e-9))
    z = ((lg - np.max(lg)) / t).astype(np.float32)
    e = rexp(z)
    p = (e / block_total(e)).astype(np.float32)
    if min_p and 0 < min_p < 1.0:
        # numpy 2 (NEP 50): a Python float meeting fp32 data computes in fp32
        keep = p >= np.float32(min_p) * np.max(p)
        p2 = np.where(keep, p, np.float32(0.0)).astype(np.float32)
        p = (p2 / block_total(p2)).astype(np.float32)
    return p


def fixed_masses(p):
    return (np.asarray(p, dtype=np.float32).astype(np.float64) * MASS_SCALE).astype(np.uint64)


def sample_fixed(logits, temperature, top_p, min_p, u):
    """The device sampler: engine.py:26-45 given the uniform draw ``u``."""
    lg = np.asarray(logits, dtype=np.float32).reshape(-1)
    if temperature <= 0:
        return int(np.argmax(lg))
    p = fixed_probs(lg, temperature, min_p)
    m = fixed_masses(p)
    if top_p < 1.0:
        keys = p.view(np.uint32)
        order = np.lexsort((np.arange(p.size), ~keys))     # descending, ties by index
        cum = np.cumsum(m[order], dtype=np.uint64)
        budget = np.uint64(float(np.float32(top_p)) * MASS_SCALE)   # top_p meets fp32 cumsums
        n_keep = int(np.searchsorted(cum, budget, side="right"))   # cum <= budget
        n_keep = max(n_keep, 1)
        kept = order[:n_keep]
        total = int(cum[n_keep - 1])
        target = np.uint64(min(int(np.uint64(float(u) * float(total))), total - 1))
        j = int(np.searchsorted(cum[:n_keep], target, side="right"))   # first cum > target
        return int(kept[j])
    cum = np.cumsum(m, dtype=np.uint64)
    total = int(cum[-1])
    target = np.uint64(min(int(np.uint64(float(u) * float(total))), total - 1))
    return int(np.searchsorted(cum, target, side="right"))
