"""TEST AND BASELINE INFRASTRUCTURE ONLY -- never part of the product path.

Runs the reference's own torch model, ptcg/rl/model.py `PTCGTransformer`,
on the CPU, for the bench's reference arm and CPU baseline:

- `load(ref_dir, s, tabs, blob)` imports the reference package from
  `ref_dir` (a checkout, or bench's offline install under baseline/_ref)
  with the shape constants of ptcg/rl/buffers.py patched before the model
  module is imported, and with `build_tables` / `load_text_tables` replaced
  by seeded tables (the competition SDK `cg.api` that cards.py:39 imports is
  not shipped).  The packed weights go through the PT_PARAMS -> state-dict
  name pairing of native/tools/native_weights.py:45-91.  Shapes bind at
  import, so one process serves one shape.
- `train_step(...)` returns a callable running one PPO minibatch step on the
  reference model: `forward_train`, the PPO loss gradients of the reference
  kernel (ppo_loss_compute, native/src/pufferlib.cu:1010-1248, through the
  restatement `ptcg_oracle.ppo_loss` that tests/test_gpu_ref_pin.py pins to
  that kernel), the aux losses ptcg_model4.cu:31-63 injects, autograd,
  `torch.nn.utils.clip_grad_norm_` and `torch.optim.Adam` (BASELINE's
  optimizer; the reference trainer has no torch optimizer).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)


def torch_name_map(s):
    """PT_PARAMS name -> reference torch state-dict name
    (native/tools/native_weights.py:45-91 pairs them in the same order)."""
    m = {
        "card_id_emb": "card_id_emb.weight", "attack_id_emb": "attack_id_emb.weight",
        "skill_id_emb": "skill_id_emb.weight",
        "attack_mlp_w": "attack_mlp.0.weight", "attack_mlp_b": "attack_mlp.0.bias",
        "skill_mlp_w": "skill_mlp.0.weight", "skill_mlp_b": "skill_mlp.0.bias",
        "card_ln_w": "card_mlp.0.weight", "card_ln_b": "card_mlp.0.bias",
        "card_mlp1_w": "card_mlp.1.weight", "card_mlp1_b": "card_mlp.1.bias",
        "card_mlp2_w": "card_mlp.3.weight", "card_mlp2_b": "card_mlp.3.bias",
        "zone_emb": "zone_emb.weight", "owner_emb": "owner_emb.weight",
        "token_proj_w": "token_proj.weight", "token_proj_b": "token_proj.bias",
        "readout": "readout",
        "global1_w": "global_mlp.0.weight", "global1_b": "global_mlp.0.bias",
        "global2_w": "global_mlp.2.weight", "global2_b": "global_mlp.2.bias",
        "sel_type_emb": "sel_type_emb.weight", "ctx_emb": "ctx_emb.weight",
        "dec1_w": "dec_mlp.0.weight", "dec1_b": "dec_mlp.0.bias",
        "dec2_w": "dec_mlp.2.weight", "dec2_b": "dec_mlp.2.bias",
        "bcast_w": "bcast.weight", "bcast_b": "bcast.bias",
        "lnf_w": "ln_f.weight", "lnf_b": "ln_f.bias",
        "opt_type_emb": "opt_type_emb.weight",
        "opt_card_w": "opt_card.weight", "opt_card_b": "opt_card.bias",
        "opt_attack_w": "opt_attack.weight", "opt_attack_b": "opt_attack.bias",
        "q1_w": "q_mlp.0.weight", "q1_b": "q_mlp.0.bias",
        "q2_w": "q_mlp.2.weight", "q2_b": "q_mlp.2.bias",
        "score1_w": "score_mlp.0.weight", "score1_b": "score_mlp.0.bias",
        "score2_w": "score_mlp.2.weight", "score2_b": "score_mlp.2.bias",
        "value1_w": "value_mlp.0.weight", "value1_b": "value_mlp.0.bias",
        "value2_w": "value_mlp.2.weight", "value2_b": "value_mlp.2.bias",
        "oracle_proj_w": "oracle_proj.weight", "oracle_proj_b": "oracle_proj.bias",
        "critic_readout": "critic_readout",
        "oracle_v1_w": "oracle_value_mlp.0.weight", "oracle_v1_b": "oracle_value_mlp.0.bias",
        "oracle_v2_w": "oracle_value_mlp.2.weight", "oracle_v2_b": "oracle_value_mlp.2.bias",
        "aux_hand_w": "aux_hand.weight", "aux_hand_b": "aux_hand.bias",
        "aux_prize_w": "aux_prize.weight", "aux_prize_b": "aux_prize.bias",
    }
    blk = {"ln1_w": "ln1.weight", "ln1_b": "ln1.bias", "qkv_w": "qkv.weight",
           "qkv_b": "qkv.bias", "proj_w": "proj.weight", "proj_b": "proj.bias",
           "ln2_w": "ln2.weight", "ln2_b": "ln2.bias", "ffn1_w": "ffn.0.weight",
           "ffn1_b": "ffn.0.bias", "ffn2_w": "ffn.2.weight", "ffn2_b": "ffn.2.bias"}
    for i in range(s.layers):
        for k, v in blk.items():
            m[f"b{i}_{k}"] = f"blocks.{i}.{v}"
    for k, v in blk.items():
        m[f"c0_{k}"] = f"critic_blocks.0.{v}"
    return m


def load(ref_dir, s, tabs, blob, param_table):
    """The reference's PTCGTransformer at shape `s` with weights `blob`."""
    import torch
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    import ptcg.rl.buffers as B
    B.MAX_TOKENS, B.TOK_F, B.N_CARDS = s.ltok, s.tok_f, s.n_cards
    B.MAX_OPTIONS, B.STOP, B.N_ATTACKS = s.nopt, s.nopt - 1, s.n_attacks
    B.OFFSETS, B.OBS_SIZE = B._build_offsets()
    B.UNK_CARD = s.n_cards - 1
    assert B.OBS_SIZE == s.obs_size, (B.OBS_SIZE, s.obs_size)
    import ptcg.rl.cards as Cd
    Cd.N_SKILLS = s.n_skills
    import ptcg.rl.model as M
    if M.MAX_TOKENS != s.ltok or M.N_CARDS != s.n_cards:
        raise RuntimeError("the reference model was imported at another shape in this process")
    M.build_tables = lambda: (tabs["card_static"], tabs["card_attacks"].astype(np.int64),
                              tabs["card_skills"].astype(np.int64), tabs["att_static"])
    M.load_text_tables = lambda: (tabs["card_text"], tabs["att_text"], tabs["skill_text"])
    model = M.PTCGTransformer(d=s.d, layers=s.layers, heads=s.heads, ffn=s.ffn, critic="oracle")
    sd = model.state_dict()
    names = torch_name_map(s)
    off = 0
    for name, shp in param_table(s):
        n = int(np.prod(shp))
        sd[names[name]] = torch.from_numpy(blob[off:off + n].reshape(shp).copy())
        off += n
    assert off == blob.size
    model.load_state_dict(sd)
    model.train(False)
    return model


def train_step(model, s, obs, actions, old_logp, adv, values, returns, prio, n_seg, horizon,
               lr=3e-4, max_norm=1.0, clip=0.2, vf_clip=0.2, vf_coef=0.5, ent_coef=0.01):
    """Callable: one PPO minibatch step of the reference model (see module
    docstring); returns the grad norm."""
    import torch
    import torch.nn.functional as F
    import ptcg_oracle as oracle
    cfg = oracle.cfg

    opt = torch.optim.Adam(model.parameters(), lr=lr, betas=(0.9, 0.999), eps=1e-8)
    obs_t = torch.from_numpy(obs)
    a, b = s.offsets["opt_mask"]
    mask = obs[:, a:b]
    hand_tgt, prized = oracle.aux_targets(obs_t, s)
    ret_t = torch.from_numpy(returns)

    def step():
        out = model.forward_train(obs_t)
        _, d_scores, d_values, _, _ = oracle.ppo_loss(
            out["logits"].detach().numpy(), mask, out["oracle_v"][:, 0].detach().numpy(),
            actions, old_logp, adv, values, returns, prio, n_seg, horizon, clip=clip,
            vf_clip=vf_clip, vf_coef=vf_coef, ent_coef=ent_coef)
        l_blind = cfg.AUX_VF_COEF * 0.5 * ((out["blind_v"][:, 0] - ret_t) ** 2).mean()
        l_hand = cfg.AUX_HAND_COEF * ((out["hand_pred"] - hand_tgt) ** 2).mean()
        um = out["unseen_mask"]
        tgt = prized.gather(1, out["token_ids"].long().clamp(0, s.n_cards - 1))
        cnt = max(float(um.sum()), 1.0)
        l_prize = cfg.AUX_PRIZE_COEF * (F.binary_cross_entropy_with_logits(
            out["prize_logits"], tgt, reduction="none") * um).sum() / cnt
        # illegal logits are -1e9 in the reference's forward; their gradient is 0
        sur = (out["logits"] * torch.from_numpy(d_scores)).sum() \
            + (out["oracle_v"][:, 0] * torch.from_numpy(d_values)).sum() \
            + l_blind + l_hand + l_prize
        opt.zero_grad(set_to_none=False)
        sur.backward()
        norm = torch.nn.utils.clip_grad_norm_(model.parameters(), max_norm)
        opt.step()
        return float(norm)
    return step
