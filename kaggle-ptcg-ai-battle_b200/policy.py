"""Python-side mirror of the reference's policy plug-in for this path.

`PTCGPolicy` plays the role that the ptcg Encoder/Decoder/Network vtables
(native/src/ocean.cu:5-46, native/model/ptcg_model4.cu:236-354) and the
trainer hooks around them (ppo_loss_fwd_bwd / muon_step / sample_logits /
ptcg_puff_advantage, native/src/pufferlib.cu) play for the reference, with
the torch-facing conveniences of ptcg/rl/model.py (forward_eval /
forward_policy / forward_train).  Device memory and streams are torch's; all
computation goes through the CUDA C-ABI (native.py); errors raise
`PtcgError` (the reference aborts / throws std::runtime_error).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import native
from .config import Shape, param_count, param_table
from .native import check

PRECISIONS = {"fp32": 0, "bf16": 1}


class _CudaArray:
    def __init__(self, ptr, n, dtype="<f4"):
        self.__cuda_array_interface__ = {
            "shape": (n,), "typestr": dtype, "data": (ptr, False), "version": 3,
            "strides": None}


def _p(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _f32(t, device):
    if isinstance(t, np.ndarray):
        t = torch.from_numpy(np.ascontiguousarray(t, np.float32))
    return t.to(device=device, dtype=torch.float32).contiguous()


class PTCGPolicy:
    def __init__(self, shape: Shape, precision="bf16", device=0, tables=None,
                 weights=None, rollout_rows=0, train_rows=0):
        self.lib = native.lib()
        self.shape = shape
        self.precision = precision
        self.device = torch.device("cuda", device)
        self._cs = native.PtcgShape.from_shape(shape)
        h = C.c_void_p()
        check(self.lib.ptcg_create(C.byref(self._cs), PRECISIONS[precision], device,
                                   C.byref(h)))
        self.h = h
        self.obs_size = self.lib.ptcg_obs_size(C.byref(self._cs))
        assert self.obs_size == shape.obs_size
        self.n_params = param_count(shape)
        self._hook_ref = None
        self._hook_err = None
        if tables is not None:
            self.set_tables(tables)
        if weights is not None:
            self.load_weights(weights)
        if rollout_rows or train_rows:
            self.reserve(rollout_rows, train_rows)

    # ---------------------------------------------------------------- setup
    def close(self):
        if getattr(self, "h", None):
            self.lib.ptcg_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_tables(self, t):
        arrs = [np.ascontiguousarray(t["card_static"], np.float32),
                np.ascontiguousarray(t["card_attacks"], np.int32),
                np.ascontiguousarray(t["card_skills"], np.int32),
                np.ascontiguousarray(t["att_static"], np.float32),
                np.ascontiguousarray(t["card_text"], np.float32),
                np.ascontiguousarray(t["att_text"], np.float32),
                np.ascontiguousarray(t["skill_text"], np.float32)]
        check(self.lib.ptcg_set_tables(self.h, *[a.ctypes.data_as(C.c_void_p) for a in arrs]))

    def load_weights(self, blob):
        b = np.ascontiguousarray(blob, np.float32)
        check(self.lib.ptcg_load_weights(self.h, b.ctypes.data_as(C.c_void_p), b.size))

    def save_weights(self):
        b = np.empty(self.n_params, np.float32)
        check(self.lib.ptcg_save_weights(self.h, b.ctypes.data_as(C.c_void_p), b.size))
        return b

    # files: packed fp32 weight blobs and PTCGSTA1 / PTCGADM1 state files
    def save_weights_file(self, path):
        check(self.lib.ptcg_save_weights_file(self.h, str(path).encode()))

    def load_weights_file(self, path):
        check(self.lib.ptcg_load_weights_file(self.h, str(path).encode()))

    def save_state(self, path, global_step=0, epoch=0, fmt="PTCGADM1"):
        f = {"PTCGSTA1": 0, "PTCGADM1": 1}[fmt]
        check(self.lib.ptcg_save_state(self.h, str(path).encode(), int(global_step), int(epoch), f))

    def load_state(self, path):
        """-> (global_step, epoch) from a PTCGSTA1 or PTCGADM1 file."""
        gs, ep = C.c_long(), C.c_long()
        check(self.lib.ptcg_load_state(self.h, str(path).encode(), C.byref(gs), C.byref(ep)))
        return gs.value, ep.value

    def packed(self, which):
        """An arena (0 params, 1 grads, 2 Adam m / Muon momentum, 3 Adam v) in
        packed PT_PARAMS order (numpy)."""
        a = self.arena(which).cpu().numpy()
        return np.concatenate([a[o:o + int(np.prod(shp))] for (_, shp), o in
                               zip(param_table(self.shape), self.param_offsets())])

    def reserve(self, rollout_rows, train_rows):
        check(self.lib.ptcg_reserve(self.h, int(rollout_rows), int(train_rows)))
        self.rollout_rows, self.train_rows = rollout_rows, train_rows

    def arena(self, which):
        """torch view of an arena: 0 params, 1 grads, 2 Adam m, 3 Adam v."""
        p = C.POINTER(C.c_float)()
        n = C.c_long()
        check(self.lib.ptcg_arena(self.h, which, C.byref(p), C.byref(n)))
        ptr = C.cast(p, C.c_void_p).value
        return torch.as_tensor(_CudaArray(ptr, n.value), device=self.device)

    def param_offsets(self):
        return [self.lib.ptcg_param_offset(self.h, i) for i in range(len(param_table(self.shape)))]

    def grads_packed(self):
        """fp32 grads in packed PT_PARAMS order (numpy)."""
        g = self.arena(1).cpu().numpy()
        out = []
        for (name, shp), off in zip(param_table(self.shape), self.param_offsets()):
            n = int(np.prod(shp))
            out.append(g[off:off + n])
        return np.concatenate(out)

    @property
    def step(self):
        v = C.c_long()
        check(self.lib.ptcg_get_step(self.h, C.byref(v)))
        return v.value

    @step.setter
    def step(self, v):
        check(self.lib.ptcg_set_step(self.h, int(v)))

    # -------------------------------------------------------- encoder slots
    def forward(self, obs):
        """Rollout forward -> (N, nopt+1) = [raw scores | oracle value]."""
        obs = _f32(obs, self.device)
        out = torch.empty(obs.shape[0], self.shape.nopt + 1, device=self.device)
        check(self.lib.ptcg_forward(self.h, _p(obs), obs.shape[0], _p(out), _stream()))
        return out

    def forward_sample(self, obs, uniforms, mask=None):
        """Rollout forward with the sampler fused into its last kernel ->
        (out, actions, logprobs, values); the same values as forward()
        followed by sample() on the obs rows' option mask (or `mask`)."""
        obs = _f32(obs, self.device)
        u = _f32(uniforms, self.device)
        n = obs.shape[0]
        out = torch.empty(n, self.shape.nopt + 1, device=self.device)
        act = torch.empty(n, device=self.device)
        logp = torch.empty(n, device=self.device)
        val = torch.empty(n, device=self.device)
        m = _f32(mask, self.device) if mask is not None else None
        check(self.lib.ptcg_forward_sample(self.h, _p(obs), n, _p(m),
                                           m.stride(0) if m is not None else 0, _p(u), _p(out),
                                           _p(act), _p(logp), _p(val), _stream()))
        return out, act, logp, val

    def obs_unpack(self, packed, out=None):
        """Compact rows (device uint8 tensor, n x ptcg_obs_packed_bytes, see
        native.obs_pack) -> fp32 observation rows on the device."""
        n = packed.shape[0]
        if out is None:
            out = torch.empty(n, self.obs_size, device=self.device)
        check(self.lib.ptcg_obs_unpack(C.byref(self._cs), _p(packed), n, _p(out), _stream()))
        return out

    def forward_eval(self, obs):
        """(masked logits (-1e9 on illegal slots), oracle value) like
        PTCGTransformer.forward_eval (ptcg/rl/model.py:315-321)."""
        obs = _f32(obs, self.device)
        out = self.forward(obs)
        a, b = self.shape.offsets["opt_mask"]
        logits = out[:, :-1].masked_fill(obs[:, a:b] == 0, -1e9)
        return logits, out[:, -1]

    def forward_policy(self, obs):
        return self.forward_eval(obs)[0]

    def forward_train(self, obs):
        obs = _f32(obs, self.device)
        self._train_obs = obs            # keep alive for backward
        out = torch.empty(obs.shape[0], self.shape.nopt + 1, device=self.device)
        check(self.lib.ptcg_forward_train(self.h, _p(obs), obs.shape[0], _p(out), _stream()))
        return out

    def backward(self, grad, returns, aux_norm_rows=0, prize_count=0.0, accumulate=False,
                 last=True):
        """Backward of the last forward_train.  accumulate adds into the grad
        arena; last=False marks a micro-batch that more of the same step
        follow, so the grad hook waits for the final one."""
        grad = _f32(grad, self.device)
        returns = _f32(returns, self.device)
        self._hook_err = None
        flags = (1 if accumulate else 0) | (0 if last else 2)
        check(self.lib.ptcg_backward(self.h, _p(grad), _p(returns), int(aux_norm_rows),
                                     float(prize_count), flags, _stream()))
        self._raise_hook_error()

    # -------------------------------------------------------- trainer hooks
    def ppo_loss(self, dec_out, mask, actions, old_logp, advantages, values, returns,
                 prio, n_seg, horizon, clip=0.2, vf_clip=0.2, vf_coef=0.5, ent_coef=0.01):
        d = self.device
        dec_out, mask = _f32(dec_out, d), _f32(mask, d)
        args = [_f32(x, d) for x in (actions, old_logp, advantages, values, returns, prio)]
        nt = n_seg * horizon
        grad = torch.empty_like(dec_out)
        nlp = torch.empty(nt, device=d)
        ratio = torch.empty(nt, device=d)
        stats = torch.zeros(8, device=d)
        scratch = torch.empty(16 + 7 * ((nt + 7) // 8), device=d)
        check(self.lib.ptcg_ppo_loss(_p(dec_out), self.shape.nopt, _p(mask),
                                     *[_p(a) for a in args], n_seg, horizon, clip, vf_clip,
                                     vf_coef, ent_coef, _p(grad), _p(nlp), _p(ratio),
                                     _p(stats), _p(scratch), _stream()))
        return grad, nlp, ratio, stats

    def adam_step(self, lr=3e-4, betas=(0.9, 0.999), eps=1e-8, max_norm=1.0, gate=None):
        stats = torch.zeros(2, device=self.device)
        check(self.lib.ptcg_adam_step(self.h, lr, betas[0], betas[1], eps, max_norm,
                                      _p(gate), _p(stats), _stream()))
        return stats

    # ------------------------------------------------ sharded optimizer
    def sumsq(self, x, out):
        """out[0] (float64 device tensor) = sum of squares of the fp32 device
        tensor x (ptcg_sumsq)."""
        check(self.lib.ptcg_sumsq(self.h, _p(x), x.numel(), _p(out), _stream()))
        return out

    def adam_segments(self, grad_src, seg, nseg, sumsq, stats, lr=3e-4, betas=(0.9, 0.999),
                      eps=1e-8, max_norm=1.0, gate=None):
        """Adam over arena segments (ptcg_adam_segments): seg int64 device
        triples {arena offset, offset in grad_src, length}, global clip from
        sumsq (float64 device scalar)."""
        check(self.lib.ptcg_adam_segments(self.h, _p(grad_src), _p(seg), int(nseg), _p(sumsq),
                                          lr, betas[0], betas[1], eps, max_norm, _p(gate),
                                          _p(stats), _stream()))
        return stats

    def refresh_copies(self):
        check(self.lib.ptcg_refresh_copies(self.h, _stream()))

    def sharded_adam(self, group=None, lr=3e-4, betas=(0.9, 0.999), eps=1e-8, max_norm=1.0):
        """A dp.ShardedAdam over this model's arenas, installed as its grad
        hook: reduce-scatter per bucket during backward, then .step(stats)."""
        from .dp import ShardedAdam
        red = ShardedAdam(self.arena(1), self.arena(0),
                          update=lambda g, seg, n, ss, st: self.adam_segments(
                              g, seg, n, ss, st, lr=lr, betas=betas, eps=eps, max_norm=max_norm),
                          sumsq=lambda x, out: self.sumsq(x, out),
                          refresh=self.refresh_copies, group=group)
        self.set_grad_hook(red)
        return red

    def dp_init(self, group=None):
        """Turn on the library's own data-parallel exchange over NCCL
        (ptcg_dp_init): rank 0 of the torch.distributed `group` makes the
        NCCL id and broadcasts it; every rank of the group must call this.
        From then on the final gradient spans are reduce-scattered during
        backward and train_step / adam_step run the sharded Adam and the
        all-gather of the weights inside the library."""
        import torch.distributed as dist
        uid = np.zeros(128, np.uint8)
        if dist.get_rank(group) == 0:
            check(self.lib.ptcg_dp_unique_id(uid.ctypes.data_as(C.c_void_p)))
        t = torch.from_numpy(uid)
        if dist.get_backend(group) == "nccl":
            t = t.to(self.device)
        dist.broadcast(t, src=dist.get_global_rank(group, 0) if group is not None else 0,
                       group=group)
        uid = t.cpu().numpy().copy()
        check(self.lib.ptcg_dp_init(self.h, uid.ctypes.data_as(C.c_void_p),
                                    dist.get_rank(group), dist.get_world_size(group)))

    def dp_weights_agree(self, out=None):
        """int64 device tensor {min, max} over the exchange's ranks of the
        weight checksum (one collective, no host wait): equal iff every rank
        holds the same weights."""
        if out is None:
            out = torch.zeros(2, dtype=torch.int64, device=self.device)
        check(self.lib.ptcg_dp_weights_agree(self.h, _p(out), _stream()))
        return out

    def dp_finalize(self, abort=False):
        check(self.lib.ptcg_dp_finalize(self.h, int(bool(abort))))

    # ---------------------------------------------- minibatch selection
    def prio_replay(self, advantages, alpha, beta, total_agents, uniforms):
        """(idx int32, mb_prio, probs) of prioritised segment replay over
        (B, T) advantages (ptcg_prio_replay)."""
        d = self.device
        adv, u = _f32(advantages, d), _f32(uniforms, d)
        B, T = adv.shape
        n = u.numel()
        idx = torch.empty(n, dtype=torch.int32, device=d)
        mb_prio = torch.empty(n, device=d)
        probs = torch.empty(B, device=d)
        cdf = torch.empty(B, device=d)
        check(self.lib.ptcg_prio_replay(_p(adv), B, T, float(alpha), float(beta),
                                        int(total_agents), n, _p(u), _p(idx), _p(mb_prio),
                                        _p(probs), _p(cdf), _stream()))
        return idx, mb_prio, probs

    def select_copy(self, idx, obs, actions, logprobs, values, advantages, mask=None):
        """Gather segments idx of (B, T, ...) rollout arrays (ptcg_select_copy);
        returns a dict with obs, actions, logprobs, values, advantages,
        returns (= values + advantages) and mask."""
        d = self.device
        idx = idx.to(device=d, dtype=torch.int32).contiguous()
        obs = _f32(obs, d)
        B, T = obs.shape[0], obs.shape[1]
        src = [_f32(x, d) for x in (actions, logprobs, values, advantages)]
        m = _f32(mask, d) if mask is not None else None
        n = idx.numel()
        out = dict(obs=torch.empty(n, T, obs.shape[2], device=d))
        for k in ("actions", "logprobs", "values", "advantages", "returns"):
            out[k] = torch.empty(n, T, device=d)
        out["mask"] = torch.empty(n, T, m.shape[2], device=d) if m is not None else None
        check(self.lib.ptcg_select_copy(_p(idx), n, T, obs.shape[2],
                                        m.shape[2] if m is not None else 0, _p(obs),
                                        *[_p(x) for x in src], _p(m), _p(out["obs"]),
                                        _p(out["actions"]), _p(out["logprobs"]),
                                        _p(out["values"]), _p(out["advantages"]),
                                        _p(out["returns"]), _p(out["mask"]), _stream()))
        return out

    def index_copy(self, dst, idx, src):
        """dst[idx[i]] = src[i] over rows (ptcg_index_copy), in place."""
        idx = idx.to(device=self.device, dtype=torch.int32).contiguous()
        n = idx.numel()
        row = src.numel() // max(n, 1)
        check(self.lib.ptcg_index_copy(_p(dst), _p(idx), _p(src), n, row, _stream()))
        return dst

    def muon_step(self, lr=0.02, momentum=0.95, weight_decay=0.0, wd_1d=0.0, max_norm=1.5,
                  gate=None):
        """The reference trainer's Muon optimizer (ptcg_muon_step); the
        momentum is arena 2.  Returns device stats {grad norm, applied}."""
        stats = torch.zeros(2, device=self.device)
        check(self.lib.ptcg_muon_step(self.h, lr, momentum, weight_decay, wd_1d, max_norm,
                                      _p(gate), _p(stats), _stream()))
        return stats

    def sample(self, dec_out, mask, uniforms):
        d = self.device
        dec_out, mask, uniforms = _f32(dec_out, d), _f32(mask, d), _f32(uniforms, d)
        n = dec_out.shape[0]
        act = torch.empty(n, device=d)
        logp = torch.empty(n, device=d)
        val = torch.empty(n, device=d)
        check(self.lib.ptcg_sample_logits(_p(dec_out), n, self.shape.nopt, _p(mask),
                                          mask.stride(0), _p(uniforms), _p(act), _p(logp),
                                          _p(val), _stream()))
        return act, logp, val

    def advantage(self, values, rewards, dones, importance, obs, gamma=0.99, lam=0.95,
                  rho_clip=1.0, c_clip=1.0):
        d = self.device
        values, rewards, dones, importance = [_f32(x, d) for x in (values, rewards, dones, importance)]
        obs = _f32(obs, d)
        B, T = values.shape
        adv = torch.zeros(B, T, device=d)
        check(self.lib.ptcg_negamax_advantage(_p(values), _p(rewards), _p(dones), _p(importance),
                                           _p(obs), self.obs_size, self.shape.seat_col, B, T,
                                           gamma, lam, rho_clip, c_clip, _p(adv), _stream()))
        return adv

    def set_grad_hook(self, fn):
        """fn(offset, count, stream_ptr) called when arena floats
        [offset, offset+count) hold final grads (last micro-batch)."""
        if fn is None:
            self._hook_ref = None
            check(self.lib.ptcg_set_grad_hook(self.h, native.GRAD_HOOK(), None))
            return
        def call(user, off, cnt, stream):
            # ctypes drops exceptions raised in callbacks: keep the first one
            # and re-raise it when the library call that fired the hook returns
            try:
                fn(off, cnt, stream)
            except BaseException as e:   # noqa: BLE001
                if self._hook_err is None:
                    self._hook_err = e

        cb = native.GRAD_HOOK(call)
        self._hook_ref = cb
        check(self.lib.ptcg_set_grad_hook(self.h, cb, None))

    def _raise_hook_error(self):
        e, self._hook_err = getattr(self, "_hook_err", None), None
        if e is not None:
            raise RuntimeError("grad hook failed") from e

    def train_step(self, obs, actions, old_logp, advantages, values, returns, prio,
                   n_seg, horizon, clip=0.2, vf_clip=0.2, vf_coef=0.5, ent_coef=0.01,
                   lr=3e-4, betas=(0.9, 0.999), eps=1e-8, max_norm=1.0, skip_adam=False,
                   stats=None):
        d = self.device
        obs = _f32(obs, d)
        args = [_f32(x, d) for x in (actions, old_logp, advantages, values, returns, prio)]
        if stats is None:
            stats = torch.zeros(16, device=d)
        self._hook_err = None
        check(self.lib.ptcg_train_step(self.h, _p(obs), *[_p(a) for a in args], n_seg,
                                       horizon, clip, vf_clip, vf_coef, ent_coef, lr, betas[0],
                                       betas[1], eps, max_norm, int(skip_adam), _p(stats),
                                       _stream()))
        self._raise_hook_error()
        return stats

    def kernel_timer(self, mode):
        """mode 1 = tcgen05 GEMM, 2 = SIMT GEMM, 3 = both, 4 = the optimizer
        kernels of adam_step, 0 = off (resets counters)."""
        check(self.lib.ptcg_kernel_timer(self.h, int(mode)))

    def kernel_timer_read(self):
        ms, n, fl = C.c_double(), C.c_long(), C.c_double()
        check(self.lib.ptcg_kernel_timer_read(self.h, C.byref(ms), C.byref(n), C.byref(fl)))
        return ms.value, n.value, fl.value

    def kernel_timer_bytes(self):
        """Algorithmic HBM bytes of the launches timed since kernel_timer(mode)."""
        b = C.c_double()
        check(self.lib.ptcg_kernel_timer_bytes(self.h, C.byref(b)))
        return b.value

    def kernel_timer_entries(self, max_entries=100000):
        """[(ms, M, N, K, a_kmajor, b_kmajor, act, engine, dtype)] of the timed launches."""
        ms = np.zeros(max_entries, np.float32)
        meta = np.zeros(8 * max_entries, np.int32)
        n = self.lib.ptcg_kernel_timer_entries(self.h, max_entries, ms.ctypes.data_as(C.c_void_p),
                                               meta.ctypes.data_as(C.c_void_p))
        if n < 0:
            check(n)
        meta = meta[:8 * n].reshape(n, 8)
        return [(float(ms[i]), *[int(v) for v in meta[i]]) for i in range(n)]

    def weights_checksum(self):
        out = torch.zeros(4, dtype=torch.int32, device=self.device)
        check(self.lib.ptcg_weights_checksum(self.h, _p(out), _stream()))
        return out[:2]
