"""The PufferLib plug-in face (include/ptcg_puffer.h) driven the way the
reference's native trainer drives its policy, through the function pointers
alone:

  create_weights -> reg_params -> reg_train / reg_rollout (x2 buffers)
  -> alloc_create of the params / grads / activation arenas
  -> ptcg_bind_train_graph -> init_weights ($PTCG_INIT_WEIGHTS)
  -> forward (rollout, train) -> decoder / network / encoder backward

(native/src/pufferlib.cu:2607-2704, native/src/models.cu:779-830).  The
Allocator bookkeeping of native/src/kernels.cu:454-466 is restated here in
Python.  Results must equal PTCGPolicy on the same weights: forwards bit for
bit, gradients within the fp32 / bf16 tolerances (unordered atomics).
"""
import ctypes as C
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

P = C.c_void_p


class Tensor(C.Structure):
    _fields_ = [("data", C.c_void_p), ("shape", C.c_int64 * 8)]


class AllocEntry(C.Structure):
    _fields_ = [("data_ptr", C.POINTER(C.c_void_p)), ("shape", C.POINTER(C.c_int64)),
                ("elem_size", C.c_int)]


class Allocator(C.Structure):
    _fields_ = [("regs", C.POINTER(AllocEntry)), ("num_regs", C.c_int), ("mem", C.c_void_p),
                ("total_elems", C.c_long), ("total_bytes", C.c_long)]


FWD = C.CFUNCTYPE(Tensor, P, P, Tensor, P)
ENC_BWD = C.CFUNCTYPE(None, P, P, Tensor, P)
DEC_BWD = C.CFUNCTYPE(Tensor, P, P, Tensor, Tensor, Tensor, P)
NET_FWD = C.CFUNCTYPE(Tensor, P, Tensor, Tensor, P, P)
NET_BWD = C.CFUNCTYPE(Tensor, P, Tensor, P, P)
INIT = C.CFUNCTYPE(None, P, C.POINTER(C.c_ulong), P)
REG_PARAMS = C.CFUNCTYPE(None, P, C.POINTER(Allocator))
REG_TRAIN = C.CFUNCTYPE(None, P, P, C.POINTER(Allocator), C.POINTER(Allocator), C.c_int)
REG_ROLL = C.CFUNCTYPE(None, P, P, C.POINTER(Allocator), C.c_int)
CREATE = C.CFUNCTYPE(P, P)
FREE = C.CFUNCTYPE(None, P)
_COMMON = [("init_weights", INIT), ("reg_params", REG_PARAMS), ("reg_train", REG_TRAIN),
           ("reg_rollout", REG_ROLL), ("create_weights", CREATE), ("free_weights", FREE),
           ("free_activations", FREE)]


class Encoder(C.Structure):
    _fields_ = [("forward", FWD), ("backward", ENC_BWD)] + _COMMON + [
        ("in_dim", C.c_int), ("out_dim", C.c_int), ("activation_size", C.c_size_t)]


class Decoder(C.Structure):
    _fields_ = [("forward", FWD), ("backward", DEC_BWD)] + _COMMON + [
        ("hidden_dim", C.c_int), ("output_dim", C.c_int), ("continuous", C.c_bool),
        ("activation_size", C.c_int)]


class Network(C.Structure):
    _fields_ = [("forward", NET_FWD), ("forward_train", NET_FWD), ("backward", NET_BWD)] + \
        _COMMON + [("hidden", C.c_int), ("num_layers", C.c_int), ("horizon", C.c_int)]


_libc = C.CDLL(None)
_libc.calloc.restype = P
_libc.calloc.argtypes = [C.c_size_t, C.c_size_t]
_libc.free.argtypes = [P]


def _numel(shape):
    n, any_ = 1, False
    for d in shape:
        if d == 0:
            break
        n *= d
        any_ = True
    return n if any_ else 0


def alloc_create(a):
    """native/src/kernels.cu:454-466: one zeroed block, each tensor at the
    next 16-byte boundary."""
    buf = torch.zeros(max(a.total_bytes, 16), dtype=torch.uint8, device="cuda")
    base, off = buf.data_ptr(), 0
    for i in range(a.num_regs):
        e = a.regs[i]
        off = (off + 15) & ~15
        e.data_ptr[0] = base + off
        off += _numel([e.shape[k] for k in range(8)]) * e.elem_size
    a.mem = base
    return buf


def tensor(t, shape=None):
    x = Tensor()
    x.data = t.data_ptr() if t is not None else None
    for k, d in enumerate(shape if shape is not None else t.shape):
        x.shape[k] = d
    return x


def view(ptr, n):
    class A:
        __cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False),
                                    "version": 3, "strides": None}
    return torch.as_tensor(A(), device="cuda")


def rel(a, b):
    a = a.double().ravel(); b = b.double().ravel()
    return float((a - b).norm() / max(b.norm(), 1e-30))


@pytest.mark.parametrize("prec", ["fp32", "bf16"])
def test_plugin_vtables_match_policy(pkg, tmp_path, prec):
    import ptcg_b200.native as native
    lib = native.lib()
    for name, res, args in (
            ("ptcg_puf_configure", C.c_int, [C.POINTER(native.PtcgShape), C.c_int, C.c_int]),
            ("ptcg_puf_set_tables", C.c_int, [P] * 7),
            ("ptcg_puf_fill_encoder", None, [C.POINTER(Encoder)]),
            ("ptcg_puf_fill_decoder", None, [C.POINTER(Decoder)]),
            ("ptcg_puf_fill_network", None, [C.POINTER(Network)]),
            ("ptcg_puf_set_abort", None, [C.c_int]),
            ("ptcg_puf_last_error", C.c_char_p, []),
            ("ptcg_bind_train_graph", None, [P]),
            ("ptcg_puff_advantage", None, [C.POINTER(Tensor)] * 6 + [C.c_float] * 4 + [P])):
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    lib.ptcg_puf_set_abort(0)
    s = pkg.config.PRESETS["tiny"]
    B, B_TT = 6, 12
    tabs = pkg.synth.make_tables(s, 11)
    blob = pkg.synth.make_weights(s, 21)
    cs = native.PtcgShape.from_shape(s)
    assert lib.ptcg_puf_configure(C.byref(cs), {"fp32": 0, "bf16": 1}[prec], 0) == 0
    t_arrs = [np.ascontiguousarray(tabs[k], np.float32 if tabs[k].dtype.kind == "f" else np.int32)
              for k in ("card_static", "card_attacks", "card_skills", "att_static", "card_text",
                        "att_text", "skill_text")]
    assert lib.ptcg_puf_set_tables(*[a.ctypes.data_as(P) for a in t_arrs]) == 0

    enc, dec, net = Encoder(), Decoder(), Network()
    lib.ptcg_puf_fill_encoder(C.byref(enc))
    lib.ptcg_puf_fill_decoder(C.byref(dec))
    lib.ptcg_puf_fill_network(C.byref(net))
    # policy_weights_create / policy_reg_train / policy_reg_rollout
    w, dw, nw = enc.create_weights(None), dec.create_weights(None), net.create_weights(None)
    params, acts, grads = Allocator(), Allocator(), Allocator()
    enc.reg_params(w, C.byref(params))
    dec.reg_params(dw, C.byref(params))
    net.reg_params(nw, C.byref(params))
    tr_enc = _libc.calloc(1, enc.activation_size)
    tr_dec = _libc.calloc(1, dec.activation_size)
    tr_net = _libc.calloc(1, 64)
    enc.reg_train(w, tr_enc, C.byref(acts), C.byref(grads), B_TT)
    dec.reg_train(dw, tr_dec, C.byref(acts), C.byref(grads), B_TT)
    net.reg_train(nw, tr_net, C.byref(acts), C.byref(grads), B_TT)
    ro = [_libc.calloc(1, enc.activation_size) for _ in range(2)]
    for r in ro:
        enc.reg_rollout(w, r, C.byref(acts), B)
    bufs = [alloc_create(a) for a in (params, grads, acts)]
    assert params.total_bytes // 4 >= blob.size
    # TrainGraph: member 6 is mb_returns (native/src/pufferlib.cu:116-129)
    rng = np.random.default_rng(4)
    ret = torch.from_numpy(rng.standard_normal(B_TT).astype(np.float32)).cuda()
    tg = (Tensor * 12)()
    tg[6] = tensor(ret)
    lib.ptcg_bind_train_graph(C.cast(tg, P))
    path = tmp_path / "init.bin"
    blob.tofile(path)
    os.environ["PTCG_INIT_WEIGHTS"] = str(path)
    stream = torch.cuda.current_stream().cuda_stream
    seed = C.c_ulong(42)
    enc.init_weights(w, C.byref(seed), stream)
    dec.init_weights(dw, C.byref(seed), stream)
    net.init_weights(nw, C.byref(seed), stream)
    assert lib.ptcg_puf_last_error() == b"", lib.ptcg_puf_last_error()

    pol = pkg.PTCGPolicy(s, precision=prec, tables=tabs, weights=blob, rollout_rows=B,
                         train_rows=B_TT)
    # the trainer's params arena holds the packed blob at the model's offsets
    par = bufs[0].view(torch.float32)
    off = pol.param_offsets()
    flat = np.concatenate([par[o:o + int(np.prod(shp))].cpu().numpy()
                           for o, (_, shp) in zip(off, pkg.config.param_table(s))])
    assert np.array_equal(flat, blob)

    # rollout forwards, one per buffer (its own workspace), bit for bit
    for k, r in enumerate(ro):
        obs = torch.from_numpy(pkg.synth.make_obs(s, B, 30 + k, edge=True)).cuda()
        o = enc.forward(w, r, tensor(obs), stream)
        h = net.forward(nw, o, Tensor(), r, stream)
        out = dec.forward(dw, r, h, stream)
        assert tuple(out.shape[:2]) == (B, s.nopt + 1)
        got = view(out.data, B * (s.nopt + 1)).view(B, -1)
        assert torch.equal(got, pol.forward(obs)), k
    # train forward, bit for bit with the policy's train path
    obs_t = torch.from_numpy(pkg.synth.make_obs(s, B_TT, 40, edge=True)).cuda()
    o = enc.forward(w, tr_enc, tensor(obs_t), stream)
    got_t = view(o.data, B_TT * (s.nopt + 1)).view(B_TT, -1).clone()
    assert torch.equal(got_t, pol.forward_train(obs_t))
    # decoder backward assembles [grad_logits | grad_value]
    gl = torch.from_numpy(rng.standard_normal((B_TT, s.nopt)).astype(np.float32) * 0.1).cuda()
    gv = torch.from_numpy(rng.standard_normal(B_TT).astype(np.float32) * 0.1).cuda()
    g = dec.backward(dw, tr_dec, tensor(gl), Tensor(), tensor(gv), stream)
    g = net.backward(nw, g, tr_net, stream)
    gcat = view(g.data, B_TT * (s.nopt + 1)).view(B_TT, -1)
    assert torch.equal(gcat, torch.cat([gl, gv[:, None]], 1))
    enc.backward(w, tr_enc, g, stream)
    assert lib.ptcg_puf_last_error() == b"", lib.ptcg_puf_last_error()
    pol.backward(torch.cat([gl, gv[:, None]], 1), ret)
    n_ar = off[-1] + int(np.prod(pkg.config.param_table(s)[-1][1]))
    g_tr = bufs[1].view(torch.float32)[:n_ar]
    g_pol = pol.arena(1)[:n_ar]
    assert rel(g_tr, g_pol) <= (1e-5 if prec == "fp32" else 2e-3), rel(g_tr, g_pol)

    # the trainer's optimizer steps its own params arena: the next train
    # forward and the next rollout forward (after a backward) see the update
    par[:n_ar] += 1e-3 * torch.randn(n_ar, device="cuda")
    torch.cuda.synchronize()
    new = np.concatenate([par[o:o + int(np.prod(shp))].cpu().numpy()
                          for o, (_, shp) in zip(off, pkg.config.param_table(s))])
    pol2 = pkg.PTCGPolicy(s, precision=prec, tables=tabs, weights=new, rollout_rows=B,
                          train_rows=B_TT)
    o = enc.forward(w, ro[1], tensor(obs_t[:B]), stream)
    assert torch.equal(view(o.data, B * (s.nopt + 1)).view(B, -1), pol2.forward(obs_t[:B]))
    o = enc.forward(w, tr_enc, tensor(obs_t), stream)
    assert torch.equal(view(o.data, B_TT * (s.nopt + 1)).view(B_TT, -1),
                       pol2.forward_train(obs_t))

    # ptcg_puff_advantage with the reference's PrecisionTensor signature
    Ba, T = 3, 8
    obs_a = torch.from_numpy(pkg.synth.make_obs(s, Ba * T, 5)).cuda().view(Ba, T, -1)
    vals, rew = [torch.from_numpy(rng.standard_normal((Ba, T)).astype(np.float32)).cuda()
                 for _ in range(2)]
    dones = torch.from_numpy((rng.random((Ba, T)) < 0.15).astype(np.float32)).cuda()
    imp = torch.from_numpy(rng.uniform(0.5, 1.5, (Ba, T)).astype(np.float32)).cuda()
    adv = torch.zeros(Ba, T, device="cuda")
    ts = [tensor(x) for x in (vals, rew, dones, imp, obs_a, adv)]
    lib.ptcg_puff_advantage(*[C.byref(t) for t in ts], 0.99, 0.95, 1.0, 1.0, stream)
    assert lib.ptcg_puf_last_error() == b"", lib.ptcg_puf_last_error()
    ref = pol.advantage(vals, rew, dones, imp, obs_a, 0.99, 0.95, 1.0, 1.0)
    assert torch.equal(adv, ref)

    torch.cuda.synchronize()
    for r in ro + [tr_enc]:
        enc.free_activations(r)
    dec.free_activations(tr_dec)
    net.free_activations(tr_net)
    enc.free_weights(w)
    dec.free_weights(dw)
    net.free_weights(nw)
    for a in (params, acts, grads):
        _libc.free(C.cast(a.regs, P))
    del os.environ["PTCG_INIT_WEIGHTS"]
