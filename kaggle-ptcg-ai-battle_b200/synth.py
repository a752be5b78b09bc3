"""Seeded synthetic inputs with the shapes and value distributions of the
BASELINE configs (there is no public dataset; these stand in for real
self-play rows).

Everything here is plain numpy with `numpy.random.default_rng(seed)`, so the
same seed produces the same arrays on every machine; the golden fixtures under
tests/golden/ are regenerated from seeds instead of being stored.

Observation rows follow the flat fp32 layout of ptcg/rl/buffers.py:212-237
(ids stored as exact floats).  Zone 0 marks padding (ptcg/rl/model.py:239),
so valid tokens draw their zone from [1, 16) and form a contiguous prefix.
"""
from __future__ import annotations

import numpy as np

from .config import (Shape, param_table, N_ZONES, N_OWNERS, N_OPT_TYPES,
                     N_SELECT_TYPES, N_CONTEXTS, TOK_INT, OPT_INT, OPT_F,
                     GLOBAL_F, DEC_F, ORACLE_HAND, ORACLE_SPLIT, ORACLE_PRIZE,
                     CARD_STATIC_F, ATTACK_STATIC_F, CARD_TEXT_F,
                     ATTACK_TEXT_F, SKILL_TEXT_F, MAX_ATTACKS, MAX_SKILLS,
                     SEAT_GLOBAL_IDX)


def make_obs(s: Shape, n: int, seed: int, edge: bool = False) -> np.ndarray:
    """(n, obs_size) float32 observation rows.

    edge=True additionally plants out-of-range / fractional ids that the
    reference clamps (native/model/ptcg_model.cu:289-344, model.py:211-233):
    negative and >= vocab card/attack/type ids, fractional ids, pointers
    beyond LTOK, zones and owners above their embedding size.
    """
    rng = np.random.default_rng(seed)
    off = s.offsets
    obs = np.zeros((n, s.obs_size), np.float32)
    lo = int(np.ceil(0.6 * s.ltok))
    hi = max(lo, int(np.floor(0.9 * s.ltok)))
    for r in range(n):
        row = obs[r]
        nv = int(rng.integers(lo, hi + 1))
        ti = np.zeros((s.ltok, TOK_INT), np.float32)
        ti[:nv, 0] = rng.integers(0, s.n_cards, nv)
        ti[:nv, 1] = rng.integers(1, N_ZONES, nv)
        ti[:nv, 2] = rng.integers(0, 2, nv)
        for c in (3, 4):
            tools = rng.integers(1, s.n_cards, nv)
            tools[rng.random(nv) < 0.5] = 0
            ti[:nv, c] = tools
        tf = np.zeros((s.ltok, s.tok_f), np.float32)
        tf[:nv] = rng.standard_normal((nv, s.tok_f))
        oi = np.zeros((s.nopt, OPT_INT), np.float32)
        oi[:, 0] = rng.integers(0, N_OPT_TYPES, s.nopt)
        for c in (1, 2):
            p = rng.integers(1, nv + 1, s.nopt)
            p[rng.random(s.nopt) < 0.3] = 0
            oi[:, c] = p
        oi[:, 3] = rng.integers(0, s.n_cards, s.nopt)
        oi[:, 4] = rng.integers(0, s.n_attacks, s.nopt)
        oi[:, 5] = rng.integers(0, 30, s.nopt)
        of = rng.standard_normal((s.nopt, OPT_F)).astype(np.float32)
        k = int(rng.integers(1, s.nopt + 1))
        mask = np.zeros(s.nopt, np.float32)
        mask[rng.choice(s.nopt, k, replace=False)] = 1.0
        gf = rng.standard_normal(GLOBAL_F).astype(np.float32)
        gf[SEAT_GLOBAL_IDX] = float(rng.integers(0, 2))
        gf[54] = 0.0      # FROZEN_ACTOR: learner rows only
        di = np.array([rng.integers(0, N_SELECT_TYPES), rng.integers(0, N_CONTEXTS),
                       rng.integers(0, s.n_cards), rng.integers(0, s.n_cards),
                       rng.integers(0, s.n_attacks), rng.integers(0, s.n_attacks),
                       rng.integers(0, s.n_cards), rng.integers(0, s.n_cards)],
                      np.float32)
        dfl = rng.standard_normal(DEC_F).astype(np.float32)
        orc = []
        cnts = np.array([0.25, 0.5, 0.75, 1.0], np.float32)
        for nslot, nf in ((ORACLE_HAND, 1), (ORACLE_SPLIT, 2), (ORACLE_PRIZE, 1)):
            ids = rng.integers(0, s.n_cards, nslot).astype(np.float32)
            ids[rng.random(nslot) < 0.3] = 0
            f = cnts[rng.integers(0, 4, (nslot, nf))]
            orc.append(np.concatenate([ids[:, None], f], 1).ravel())
        orc = np.concatenate(orc)
        if edge:
            ti[0, 0] = s.n_cards + 5          # clamps to NC-1
            ti[1 % nv, 0] = -3                # clamps to 0
            ti[2 % nv, 0] = 7.6               # truncates to 7
            ti[0, 1] = N_ZONES + 4            # valid, embedding clamps to 15
            ti[1 % nv, 2] = N_OWNERS + 3      # owner clamps to 3
            ti[3 % nv, 2] = -2                # owner clamps to 0
            ti[0, 3] = s.n_cards + 11         # tool clamps to NC-1
            ti[1 % nv, 4] = -5                # tool ignored (not > 0)
            oi[0, 0] = N_OPT_TYPES + 9
            oi[1, 0] = -1
            oi[0, 1] = s.ltok + 3             # pointer out of range -> zeros
            oi[1, 2] = -4                     # pointer <= 0 -> zeros
            oi[0, 3] = s.n_cards + 2
            oi[1, 4] = s.n_attacks + 1
            oi[2 % s.nopt, 4] = -7
            di[0] = N_SELECT_TYPES + 3
            di[1] = -1
            di[2] = s.n_cards * 2
            di[4] = -2
            di[5] = s.n_attacks + 5
            orc[0] = s.n_cards + 3            # hand id out of range
            orc[2] = -1
        a, b = off["tok_int"]; row[a:b] = ti.ravel()
        a, b = off["tok_float"]; row[a:b] = tf.ravel()
        a, b = off["opt_int"]; row[a:b] = oi.ravel()
        a, b = off["opt_float"]; row[a:b] = of.ravel()
        a, b = off["opt_mask"]; row[a:b] = mask
        a, b = off["global_f"]; row[a:b] = gf
        a, b = off["dec_int"]; row[a:b] = di
        a, b = off["dec_float"]; row[a:b] = dfl
        a, b = off["oracle"]; row[a:b] = orc
    return obs


def make_obs_batch(s: Shape, n: int, seed: int) -> np.ndarray:
    """Vectorised `make_obs` (same distributions, its own random stream) for
    minibatch-sized inputs."""
    rng = np.random.default_rng(seed)
    off = s.offsets
    obs = np.zeros((n, s.obs_size), np.float32)
    lo = int(np.ceil(0.6 * s.ltok))
    hi = max(lo, int(np.floor(0.9 * s.ltok)))
    nv = rng.integers(lo, hi + 1, n)
    valid = np.arange(s.ltok)[None, :] < nv[:, None]                  # (n, ltok)
    ti = np.zeros((n, s.ltok, TOK_INT), np.float32)
    ti[:, :, 0] = rng.integers(0, s.n_cards, (n, s.ltok))
    ti[:, :, 1] = rng.integers(1, N_ZONES, (n, s.ltok))
    ti[:, :, 2] = rng.integers(0, 2, (n, s.ltok))
    for c in (3, 4):
        t = rng.integers(1, s.n_cards, (n, s.ltok))
        t[rng.random((n, s.ltok)) < 0.5] = 0
        ti[:, :, c] = t
    ti *= valid[:, :, None]
    tf = rng.standard_normal((n, s.ltok, s.tok_f)).astype(np.float32) * valid[:, :, None]
    oi = np.zeros((n, s.nopt, OPT_INT), np.float32)
    oi[:, :, 0] = rng.integers(0, N_OPT_TYPES, (n, s.nopt))
    for c in (1, 2):
        p = np.floor(rng.random((n, s.nopt)) * nv[:, None]).astype(np.int64) + 1
        p[rng.random((n, s.nopt)) < 0.3] = 0
        oi[:, :, c] = p
    oi[:, :, 3] = rng.integers(0, s.n_cards, (n, s.nopt))
    oi[:, :, 4] = rng.integers(0, s.n_attacks, (n, s.nopt))
    oi[:, :, 5] = rng.integers(0, 30, (n, s.nopt))
    of = rng.standard_normal((n, s.nopt, OPT_F)).astype(np.float32)
    k = rng.integers(1, s.nopt + 1, n)
    rank = np.argsort(rng.random((n, s.nopt)), axis=1).argsort(axis=1)
    mask = (rank < k[:, None]).astype(np.float32)                      # k random legal slots
    gf = rng.standard_normal((n, GLOBAL_F)).astype(np.float32)
    gf[:, SEAT_GLOBAL_IDX] = rng.integers(0, 2, n)
    gf[:, 54] = 0.0
    di = np.stack([rng.integers(0, N_SELECT_TYPES, n), rng.integers(0, N_CONTEXTS, n),
                   rng.integers(0, s.n_cards, n), rng.integers(0, s.n_cards, n),
                   rng.integers(0, s.n_attacks, n), rng.integers(0, s.n_attacks, n),
                   rng.integers(0, s.n_cards, n), rng.integers(0, s.n_cards, n)],
                  1).astype(np.float32)
    dfl = rng.standard_normal((n, DEC_F)).astype(np.float32)
    cnts = np.array([0.25, 0.5, 0.75, 1.0], np.float32)
    parts = []
    for nslot, nf in ((ORACLE_HAND, 1), (ORACLE_SPLIT, 2), (ORACLE_PRIZE, 1)):
        ids = rng.integers(0, s.n_cards, (n, nslot)).astype(np.float32)
        ids[rng.random((n, nslot)) < 0.3] = 0
        f = cnts[rng.integers(0, 4, (n, nslot, nf))]
        parts.append(np.concatenate([ids[:, :, None], f], 2).reshape(n, -1))
    orc = np.concatenate(parts, 1)
    for name, v in (("tok_int", ti), ("tok_float", tf), ("opt_int", oi), ("opt_float", of),
                    ("opt_mask", mask), ("global_f", gf), ("dec_int", di),
                    ("dec_float", dfl), ("oracle", orc)):
        a, b = off[name]
        obs[:, a:b] = v.reshape(n, -1)
    return obs


def sample_legal(mask: np.ndarray, seed: int) -> np.ndarray:
    """One uniformly drawn legal slot per row (float32 action ids)."""
    rng = np.random.default_rng(seed)
    r = rng.random(mask.shape) * (mask != 0)
    return r.argmax(1).astype(np.float32)


def make_tables(s: Shape, seed: int):
    """Seeded stand-ins for the engine-derived static tables
    (ptcg/rl/cards.py:39-82) and the text-embedding channels
    (cards.py:28-36).  The competition SDK (`cg.api`) is not shipped."""
    rng = np.random.default_rng(seed)
    card_static = rng.random((s.n_cards, CARD_STATIC_F)).astype(np.float32)
    card_attacks = rng.integers(0, s.n_attacks, (s.n_cards, MAX_ATTACKS)).astype(np.int32)
    card_attacks[rng.random(card_attacks.shape) < 0.35] = 0
    card_skills = rng.integers(0, s.n_skills, (s.n_cards, MAX_SKILLS)).astype(np.int32)
    card_skills[rng.random(card_skills.shape) < 0.6] = 0
    att_static = rng.random((s.n_attacks, ATTACK_STATIC_F)).astype(np.float32)
    card_text = (0.3 * rng.standard_normal((s.n_cards, CARD_TEXT_F))).astype(np.float32)
    att_text = (0.3 * rng.standard_normal((s.n_attacks, ATTACK_TEXT_F))).astype(np.float32)
    skill_text = (0.3 * rng.standard_normal((s.n_skills, SKILL_TEXT_F))).astype(np.float32)
    return dict(card_static=card_static, card_attacks=card_attacks,
                card_skills=card_skills, att_static=att_static,
                card_text=card_text, att_text=att_text, skill_text=skill_text)


def make_weights(s: Shape, seed: int, std: float = 0.02) -> np.ndarray:
    """Packed fp32 blob in PT_PARAMS order: every tensor ~ N(0, std), except
    LayerNorm gains which are 1 + N(0, std) (an all-~0 gain would scale the
    whole trunk signal down by 50x and make relative parity meaningless)."""
    rng = np.random.default_rng(seed)
    chunks = []
    for name, shp in param_table(s):
        w = (std * rng.standard_normal(shp)).astype(np.float32)
        if name.endswith("ln1_w") or name.endswith("ln2_w") or name in (
                "lnf_w", "card_ln_w"):
            w += 1.0
        chunks.append(w.ravel())
    return np.concatenate(chunks).astype(np.float32)


def make_rollout_batch(s: Shape, n_seg: int, horizon: int, seed: int,
                       scores: np.ndarray | None = None):
    """PPO minibatch tensors: actions sampled from the
    legal mask (uniform over legal slots unless `scores` are given, in which
    case from the masked softmax), advantages / returns ~ N(0, 1),
    prio weights 1.  Returns a dict of (n_seg*horizon,) arrays."""
    rng = np.random.default_rng(seed)
    nt = n_seg * horizon
    return dict(
        advantages=rng.standard_normal(nt).astype(np.float32),
        returns=rng.standard_normal(nt).astype(np.float32),
        prio=np.ones(n_seg, np.float32),
        uniforms=rng.random(nt).astype(np.float32),
    )
