"""Runtime shape configuration of the PTCG policy.

The reference fixes its sizes at compile time (`PT_D/PT_H/PT_FFN/PT_LAYERS`
and friends, native/model/ptcg_model.cu:14-87) and keeps a second copy of them
in native/tools/native_weights.py:24-37.  Here every width is a runtime field
of `Shape`; the C-ABI (`include/ptcg_b200.h`, `PtcgShape`) carries the same
fields in the same order.

Derived widths follow the torch module definitions of
ptcg/rl/model.py:94-175 and the observation layout of
ptcg/rl/buffers.py:29-55, 212-237.
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass

# fixed vocabularies / widths that do not move with the BASELINE configs
# (ptcg/rl/buffers.py:58-75, ptcg/rl/model.py:94-175)
N_ZONES = 16
N_OWNERS = 4
N_OPT_TYPES = 33
N_SELECT_TYPES = 29
N_CONTEXTS = 65
TOK_INT = 5
OPT_INT = 6
OPT_F = 8
GLOBAL_F = 64
DEC_INT = 8
DEC_F = 16
ORACLE_HAND, ORACLE_SPLIT, ORACLE_PRIZE = 24, 24, 8
N_ORACLE_TOKENS = ORACLE_HAND + ORACLE_SPLIT + ORACLE_PRIZE          # 56
ORACLE_F = ORACLE_HAND * 2 + ORACLE_SPLIT * 3 + ORACLE_PRIZE * 2      # 136
CARD_STATIC_F = 58
ATTACK_STATIC_F = 15
CARD_TEXT_F, ATTACK_TEXT_F, SKILL_TEXT_F = 128, 64, 64
MAX_ATTACKS, MAX_SKILLS = 4, 2
ZONE_MY_UNSEEN = 9            # ptcg/rl/buffers.py Zone.MY_UNSEEN
SEAT_GLOBAL_IDX = 31          # GlobF.ACTOR_SEAT (buffers.py:170)
AUX_VF_COEF = 1.0             # native/model/ptcg_model.cu:85-87
AUX_HAND_COEF = 0.1
AUX_PRIZE_COEF = 0.1


@dataclass(frozen=True)
class Shape:
    d: int = 256
    heads: int = 8
    ffn: int = 1024
    layers: int = 4
    ltok: int = 128
    nopt: int = 64
    tok_f: int = 32
    n_cards: int = 4096
    n_attacks: int = 1573
    n_skills: int = 448
    d_c: int = 128
    d_a: int = 64
    g: int = 128

    # ---- derived widths (ptcg/rl/model.py / ptcg_model.cu:14-66)
    @property
    def dh(self): return self.d // self.heads
    @property
    def lseq(self): return self.ltok + 1
    @property
    def norc(self): return N_ORACLE_TOKENS
    @property
    def lcrit(self): return 1 + self.lseq + self.norc
    @property
    def att_in(self): return 48 + ATTACK_STATIC_F + ATTACK_TEXT_F          # 127
    @property
    def sk_in(self): return 48 + SKILL_TEXT_F                              # 112
    @property
    def card_in(self):
        return 64 + CARD_STATIC_F + CARD_TEXT_F + 2 * self.d_a + 2 * self.d_c  # 634
    @property
    def tok_in(self): return 2 * self.d_c + self.tok_f + 8 + 4
    @property
    def dec_in(self): return 8 + 32 + 2 * self.d_c + 2 * self.d_a + 2 * self.d_c + DEC_F
    @property
    def orc_in(self): return self.d_c + 6
    @property
    def bcast_in(self): return self.g + 64
    @property
    def q_in(self): return 16 + 2 * self.d + 64 + 64 + OPT_F
    @property
    def score_in(self): return 3 * self.d + self.g + 64
    @property
    def val_in(self): return self.d + self.g

    # ---- observation layout (ptcg/rl/buffers.py:212-237)
    def obs_sections(self):
        return [
            ("tok_int", self.ltok * TOK_INT),
            ("tok_float", self.ltok * self.tok_f),
            ("opt_int", self.nopt * OPT_INT),
            ("opt_float", self.nopt * OPT_F),
            ("opt_mask", self.nopt),
            ("global_f", GLOBAL_F),
            ("dec_int", DEC_INT),
            ("dec_float", DEC_F),
            ("oracle", ORACLE_F),
        ]

    @property
    def offsets(self):
        off, cur = {}, 0
        for name, size in self.obs_sections():
            off[name] = (cur, cur + size)
            cur += size
        return off

    @property
    def obs_size(self):
        return sum(s for _, s in self.obs_sections())

    @property
    def seat_col(self):
        return self.offsets["global_f"][0] + SEAT_GLOBAL_IDX

    def with_(self, **kw):
        return dataclasses.replace(self, **kw)


PRESETS = {
    # reference defaults (native/model/ptcg_model.cu:22-44)
    "default": Shape(d=256, heads=8, ffn=512, layers=4, ltok=160, nopt=64,
                     tok_f=56, n_cards=1284, n_attacks=1573, n_skills=448),
    # BASELINE configs 0-3
    "c0": Shape(),
    # BASELINE config 4
    "c4": Shape(d=512, heads=16, ffn=2048, layers=8, ltok=256, nopt=128),
    # small shape used for the full-gradient golden fixtures and fast tests
    "tiny": Shape(d=64, heads=2, ffn=128, layers=2, ltok=16, nopt=8, tok_f=8,
                  n_cards=64, n_attacks=40, n_skills=24),
    # mid-size shape: same widths as c0 but short sequences, for GPU parity
    "small": Shape(d=256, heads=8, ffn=1024, layers=2, ltok=32, nopt=16,
                   tok_f=32, n_cards=512, n_attacks=200, n_skills=64),
}


def block_params(prefix, s: Shape):
    d, f = s.d, s.ffn
    return [
        (prefix + "ln1_w", (d,)), (prefix + "ln1_b", (d,)),
        (prefix + "qkv_w", (3 * d, d)), (prefix + "qkv_b", (3 * d,)),
        (prefix + "proj_w", (d, d)), (prefix + "proj_b", (d,)),
        (prefix + "ln2_w", (d,)), (prefix + "ln2_b", (d,)),
        (prefix + "ffn1_w", (f, d)), (prefix + "ffn1_b", (f,)),
        (prefix + "ffn2_w", (d, f)), (prefix + "ffn2_b", (d,)),
    ]


def param_table(s: Shape):
    """(name, shape) in the packed-blob order of PT_PARAMS
    (native/model/ptcg_model.cu:95-126; native/tools/native_weights.py:45-91)."""
    d, dc, da, g = s.d, s.d_c, s.d_a, s.g
    t = [
        ("card_id_emb", (s.n_cards, 64)), ("attack_id_emb", (s.n_attacks, 48)),
        ("skill_id_emb", (s.n_skills, 48)),
        ("attack_mlp_w", (da, s.att_in)), ("attack_mlp_b", (da,)),
        ("skill_mlp_w", (dc, s.sk_in)), ("skill_mlp_b", (dc,)),
        ("card_ln_w", (s.card_in,)), ("card_ln_b", (s.card_in,)),
        ("card_mlp1_w", (256, s.card_in)), ("card_mlp1_b", (256,)),
        ("card_mlp2_w", (dc, 256)), ("card_mlp2_b", (dc,)),
        ("zone_emb", (N_ZONES, 8)), ("owner_emb", (N_OWNERS, 4)),
        ("token_proj_w", (d, s.tok_in)), ("token_proj_b", (d,)),
        ("readout", (d,)),
        ("global1_w", (g, GLOBAL_F)), ("global1_b", (g,)),
        ("global2_w", (g, g)), ("global2_b", (g,)),
        ("sel_type_emb", (N_SELECT_TYPES, 8)), ("ctx_emb", (N_CONTEXTS, 32)),
        ("dec1_w", (64, s.dec_in)), ("dec1_b", (64,)),
        ("dec2_w", (64, 64)), ("dec2_b", (64,)),
        ("bcast_w", (d, s.bcast_in)), ("bcast_b", (d,)),
    ]
    for i in range(s.layers):
        t += block_params(f"b{i}_", s)
    t += [
        ("lnf_w", (d,)), ("lnf_b", (d,)),
        ("opt_type_emb", (N_OPT_TYPES, 16)),
        ("opt_card_w", (64, dc)), ("opt_card_b", (64,)),
        ("opt_attack_w", (64, da)), ("opt_attack_b", (64,)),
        ("q1_w", (d, s.q_in)), ("q1_b", (d,)),
        ("q2_w", (d, d)), ("q2_b", (d,)),
        ("score1_w", (256, s.score_in)), ("score1_b", (256,)),
        ("score2_w", (1, 256)), ("score2_b", (1,)),
        ("value1_w", (256, s.val_in)), ("value1_b", (256,)),
        ("value2_w", (1, 256)), ("value2_b", (1,)),
        ("oracle_proj_w", (d, s.orc_in)), ("oracle_proj_b", (d,)),
        ("critic_readout", (d,)),
    ]
    t += block_params("c0_", s)
    t += [
        ("oracle_v1_w", (256, s.val_in)), ("oracle_v1_b", (256,)),
        ("oracle_v2_w", (1, 256)), ("oracle_v2_b", (1,)),
        ("aux_hand_w", (s.n_cards, s.val_in)), ("aux_hand_b", (s.n_cards,)),
        ("aux_prize_w", (1, d)), ("aux_prize_b", (1,)),
    ]
    return t


def param_count(s: Shape):
    n = 0
    for _, shp in param_table(s):
        k = 1
        for x in shp:
            k *= x
        n += k
    return n


def packed_offsets(s: Shape):
    """name -> (offset, shape) in the packed fp32 blob."""
    out, off = {}, 0
    for name, shp in param_table(s):
        k = 1
        for x in shp:
            k *= x
        out[name] = (off, shp)
        off += k
    return out


def forward_flops(s: Shape, critic_rows: str = "first"):
    """Dense multiply-add FLOPs (2 per MAC) of one sample's policy forward at
    the full padded lengths LSEQ / LCRIT, by part.  ``critic_rows="all"``
    counts the critic block over every row, as the reference executes it
    (ptcg_model3.cu:333-355); ``"first"`` counts what this build runs: the
    critic output is read at its readout row only (model.py:305-308), so its
    QKV covers every row (keys / values) and attention, proj and FFN cover
    row 0.  Static-table MLPs are per call, not per sample, and excluded."""
    D, F = s.d, s.ffn

    def block(L, rows_out):
        qkv = 2 * L * 3 * D * D
        att = 4 * rows_out * L * D                    # QK^T and PV
        post = 2 * rows_out * (D * D + 2 * D * F)     # proj + FFN
        return qkv + att + post

    L, LC = s.lseq, s.lcrit
    parts = {
        "token_proj": 2 * s.ltok * s.tok_in * D,
        "trunk": s.layers * block(L, L),
        "critic": block(LC, LC if critic_rows == "all" else 1)
        + 2 * N_ORACLE_TOKENS * s.orc_in * D + 2 * s.val_in * 256 + 2 * 256,
        "options": s.nopt * (2 * s.q_in * D + 2 * D * D + 2 * s.score_in * 256 + 2 * 256),
    }
    parts["total"] = sum(parts.values())
    return parts


def train_flops(s: Shape, critic_rows: str = "first"):
    """Per-sample train-step FLOPs: forward plus a backward of twice the
    forward (dX and dW GEMMs)."""
    return 3 * forward_flops(s, critic_rows)["total"]


def bf16_copied(name: str) -> bool:
    """Parameters whose bf16 compute copy the Adam pass refreshes in bf16
    mode: the block matrices, token_proj, oracle_proj and aux_hand."""
    block = (len(name) > 3 and name[0] in "bc" and name[1].isdigit()
             and any(k in name for k in ("qkv_w", "proj_w", "ffn1_w", "ffn2_w")))
    return block or name in ("token_proj_w", "oracle_proj_w", "aux_hand_w")


def optimizer_bytes(s: Shape, bf16: bool = True):
    """Algorithmic HBM bytes of one clip + Adam step over the arena (every
    tensor padded to 16 bytes): the norm pass reads the grads (4 B/float);
    the update reads grad, param, m, v and writes param, m, v (28 B/float)
    and writes the bf16 copies (2 B per copied parameter)."""
    import numpy as np
    arena = sum((int(np.prod(shp)) + 3) // 4 * 4 for _, shp in param_table(s))
    copied = sum(int(np.prod(shp)) for name, shp in param_table(s) if bf16 and bf16_copied(name))
    return {"norm_pass": 4 * arena, "update_pass": 28 * arena + 2 * copied,
            "total": 32 * arena + 2 * copied}
