"""Generate the golden parity fixtures by running the REFERENCE implementation.

Run in a container that has the reference checked out (it is not needed, and
not present, where the tests run):

    PRISM_REFERENCE=/path/to/Prism python tests/golden/make_golden.py

The reference's own Python code is imported unmodified, with stub parent
packages so that ``hymm/models/modules/__init__.py`` (which needs diffusers)
is skipped, ``TORCHDYNAMO_DISABLE=1`` (its @torch.compile helpers run eagerly)
and ``TRITON_INTERPRET=1`` (its Triton kernels run on CPU tensors).  Shipped
``.pyc`` files are never loaded (``sys.dont_write_bytecode`` + a private
``PYTHONPYCACHEPREFIX`` are set by the caller or below).

For every case in ``inputs.CASES`` the fixture ``<case>.npz`` stores:
* audio token norms as produced by ``a2v.norm(dim=-1)`` (wan_video_dit.py:744);
* ``g``, ``rho`` from ``compute_effective_gradient`` and ``shape_ids`` from
  ``select_zone_shapes`` (dynamic_block_shape.py:248-391) on the bf16 head mean;
* ``src_idx`` and the tile-level selection (packed bits of
  ``tile_block_indices``/``lens``, dynamic_block_attention.py:297-319) captured
  at the kernel call;
* the attention output and dQ/dK/dV of ``flash_attn_bsa_3d_dynamic`` run in
  fp32 on the same (bf16-representable) values with the captured shape ids,
  for a fixed random subset of 128 rows, plus full-tensor checksums.

Without a valid mask (grid already a multiple of 8) the reference pools and
scores in bf16 (mean_pooling_compression, bsa_interface.py:164-174), so the
bf16 pass (``sel_bits``, what the model runs) and the fp32 pass
(``sel_bits_f32``) may select differently; both are stored.
"""
from __future__ import annotations

import os
import sys
import types

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
os.environ.setdefault("TRITON_INTERPRET", "1")
os.environ.setdefault("PYTHONPYCACHEPREFIX", "/tmp/prism_pyc")
sys.dont_write_bytecode = True

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from inputs import ALL_CASES, CROSS_CASES, make_cross_inputs, make_inputs  # noqa: E402
from inputs import PRODUCER_CASES as PRODUCER_FIXTURES, make_producer_inputs  # noqa: E402

N_ROWS = 128  # output rows stored per head (a fixed random subset)


def import_reference(root):
    def stub(name, path):
        m = types.ModuleType(name)
        m.__path__ = [path]
        sys.modules[name] = m

    stub("hymm", f"{root}/hymm")
    stub("hymm.models", f"{root}/hymm/models")
    stub("hymm.models.modules", f"{root}/hymm/models/modules")
    stub("hymm.utils", f"{root}/hymm/utils")
    from hymm.models.modules.block_sparse_attention import dynamic_block_attention as dba
    from hymm.models.modules.block_sparse_attention import dynamic_block_shape as dbs
    from hymm.models.modules.block_sparse_attention import bsa_interface as bsa
    return dba, dbs, bsa


def import_bias_rectification():
    from hymm.models.modules.block_sparse_attention import bias_rectification as br
    return br


def run_case(dba, dbs, case):
    from oracle.oracle import dense_to_bits, tile_lists_to_dense

    inp = make_inputs(case)
    Tp, Hp, Wp = case.grid_padded
    S = Tp * Hp * Wp
    n_tiles = S // 64
    q, k, v, do = inp["q"], inp["k"], inp["v"], inp["do"]
    valid, norms = inp["valid"], inp["norms"]
    ZT, ZH, ZW = Tp // 8, Hp // 8, Wp // 8

    with torch.no_grad():
        vavg = v[0].mean(dim=0).view(Tp, Hp, Wp, -1)
        g, rho = dbs.compute_effective_gradient(vavg, norms, ZT, ZH, ZW, lambda_a=case.lambda_a,
                                                valid_mask_thw=valid, sp_reduce=True)

    captured = []
    orig_apply = dba._dyn_bsa_kernel.apply

    def capture_apply(q_re, k_re, v_re, sm_scale, tbi, lens, cq, ck, sp, valid_re):
        captured.append(dict(tbi=tbi.clone(), lens=lens.clone()))
        return orig_apply(q_re, k_re, v_re, sm_scale, tbi, lens, cq, ck, sp, valid_re)

    try:
        kw = dict(method=case.method, sparsity=case.sparsity, cdf_threshold=case.cdf_threshold,
                  audio_token_norms=norms, valid_mask=valid, lambda_a=case.lambda_a,
                  tau_128=case.tau_128, lambda_128=case.lambda_128)
        # pass 1: bf16 inputs -> shape choice and selection exactly as the model sees them
        # (the attention kernel itself is run in fp32 below; here only its inputs are captured)
        dba._dyn_bsa_kernel.apply = lambda *a: (captured.append(
            dict(tbi=a[4].clone(), lens=a[5].clone())) or a[0].float())
        with torch.no_grad():
            _, shape_ids = dba.flash_attn_bsa_3d_dynamic(q, k, v, case.grid_padded,
                                                         return_shape_ids=True, **kw)
        sel_bf16 = captured.pop()
        # pass 2: fp32 values (bf16-representable), cached shape ids, real kernels, autograd
        dba._dyn_bsa_kernel.apply = capture_apply
        q32, k32, v32 = (t.float().requires_grad_(True) for t in (q, k, v))
        out = dba.flash_attn_bsa_3d_dynamic(q32, k32, v32, case.grid_padded, shape_ids=shape_ids,
                                            **kw)
        (out * do.float()).sum().backward()
        sel_f32 = captured.pop()
    finally:
        dba._dyn_bsa_kernel.apply = orig_apply

    src_idx, _ = dba._build_rearrange_index(shape_ids, ZT, ZH, ZW, Hp, Wp, "cpu")
    dense16 = tile_lists_to_dense(sel_bf16["tbi"].numpy(), sel_bf16["lens"].numpy(), n_tiles)
    dense32 = tile_lists_to_dense(sel_f32["tbi"].numpy(), sel_f32["lens"].numpy(), n_tiles)
    if valid is not None:
        # masked path: pooling and scores are fp32 in both passes
        assert (dense16 == dense32).all(), "selection differs between bf16 and fp32 passes"

    res = dict(
        grid=np.array(case.grid), grid_padded=np.array(case.grid_padded),
        shape_ids=shape_ids.numpy().astype(np.int64), g=g.numpy(), rho=rho.numpy(),
        src_idx=src_idx.numpy().astype(np.int32), sel_bits=dense_to_bits(dense16),
        sel_bits_f32=dense_to_bits(dense32),
    )
    if norms is not None:
        res["norms_u"] = inp["norms_u"].view(torch.int16).numpy().view(np.uint16)
    h, D = case.heads, case.head_dim
    o = out.detach()[0].numpy()
    grads = [t.grad[0].numpy() for t in (q32, k32, v32)]
    rng = np.random.default_rng(1234)
    rows = np.sort(rng.choice(S, size=min(S, N_ROWS), replace=False))
    res["rows"] = rows.astype(np.int64)
    res["o"] = o[:, rows]
    res["dq"], res["dk"], res["dv"] = (gr[:, rows] for gr in grads)
    res["sums"] = np.array([np.abs(x).astype(np.float64).sum() for x in [o] + grads])
    return res


def chunk_lists_to_dense(block_indices, lens, n_cols):
    """Reference chunk selection (block_indices [B,h,nq,W], lens [B,h,nq]) -> [h, nq, n_cols]."""
    bi = np.asarray(block_indices)[0]
    ln = np.asarray(lens)[0]
    h, nq, w = bi.shape
    dense = np.zeros((h, nq, n_cols), bool)
    keep = np.arange(w)[None, None, :] < ln[..., None]
    hh, rr, cc = np.nonzero(keep)
    dense[hh, rr, bi[hh, rr, cc]] = True
    return dense


def _uniform_entry(bsa, case, inp, dtype):
    """The reference entry point of a uniform case as f(q, k, v, **kw) for one pass
    (dtype = the pass's floating type: guidance gains, gate and norms follow it, as
    in wan_video_dit.py:309-335 where they take q's dtype)."""
    g = case.guidance
    gp = case.grid_padded
    if g is None:
        return lambda q, k, v, **kw: bsa.flash_attn_bsa_3d(q, k, v, gp, gp, **kw)
    if g["kind"] == "variance":
        return lambda q, k, v, **kw: bsa.flash_attn_bsa_3d_variance_guided(
            q, k, v, gp, gp, variance_boost_gamma=g["variance_gamma"], **kw)
    norms = inp["norms"].to(dtype)
    gate = torch.tensor([g["gate"]], dtype=dtype)
    gamma = torch.tensor(g["audio_gamma"], dtype=dtype)
    return lambda q, k, v, **kw: bsa.flash_attn_bsa_3d_audio_guided(
        q, k, v, gp, gp, audio_token_norms=norms, audio_gate_value=gate, audio_boost_gamma=gamma,
        audio_weighted_lambda=g["lambda_w"], variance_boost_gamma=g["variance_gamma"], **kw)


def _guidance_parts(bsa, case, inp):
    """The reference's guidance statistics on fp32 values: rho
    (compute_channel_variance_density), the audio block saliency
    (compute_block_audio_saliency) and Path B's pooled keys
    (audio_weighted_mean_pooling_compression), each on the key chunk order."""
    g = case.guidance
    Tp, Hp, Wp = case.grid_padded
    tk, hk, wk = case.chunk_k
    n3 = (Tp // tk, Hp // hk, Wp // wk)
    ck = tk * hk * wk
    D = case.head_dim
    valid = inp["valid"]
    vm = None if valid is None else bsa.rearrange_THW_to_3d_block_1d(valid, *n3, tk, hk, wk)
    out = {}
    with torch.no_grad():
        if g.get("variance_gamma", 0.0) > 0:
            v_ro = bsa.rearrange_THW_to_3d_block(inp["v"].float(), *n3, tk, hk, wk, D)
            out["rho"] = bsa.compute_channel_variance_density(v_ro, ck, tk, hk, wk, vm).numpy()
        if g["kind"] == "audio":
            a_ro = bsa.rearrange_THW_to_3d_block_1d(inp["norms"].float(), *n3, tk, hk, wk)
            out["saliency"] = bsa.compute_block_audio_saliency(a_ro, ck, valid_mask=vm).numpy()
            if g["lambda_w"] > 0:
                k_ro = bsa.rearrange_THW_to_3d_block(inp["k"].float(), *n3, tk, hk, wk, D)
                kc = bsa.audio_weighted_mean_pooling_compression(k_ro, ck, a_ro, valid_mask=vm,
                                                                 lambda_w=g["lambda_w"])
                out["kcmp_pathb"] = kc[0].numpy()
    return out


def run_uniform_case(bsa, case):
    """flash_attn_bsa_3d (bsa_interface.py:1123-1176) on the padded grid, as the
    uniform dispatch of wan_video_dit.py:470-560 calls it, or its guided forms
    (flash_attn_bsa_3d_variance_guided :1179-1260, flash_attn_bsa_3d_audio_guided
    :1395-1501, dispatched at wan_video_dit.py:637-672).  Stores the chunk
    orders, the chunk-level selection of a bf16 and an fp32 pass, and the fp32
    outputs / gradients on a fixed subset of rows (padded THW order); guided cases
    add the reference's guidance statistics."""
    from oracle.oracle import dense_to_bits

    inp = make_inputs(case)
    Tp, Hp, Wp = case.grid_padded
    S = Tp * Hp * Wp
    q, k, v, do, valid = inp["q"], inp["k"], inp["v"], inp["do"], inp["valid"]
    cq, ck = case.chunk_q, case.chunk_k
    nq, nk = S // (cq[0] * cq[1] * cq[2]), S // (ck[0] * ck[1] * ck[2])
    kw = dict(sparsity=case.sparsity, cdf_threshold=case.cdf_threshold,
              chunk_3d_shape_q=list(cq), chunk_3d_shape_k=list(ck), valid_mask=valid)
    captured = []
    orig = bsa.attn_fwd_bsa_varlen_triton

    def skip(q_, k_, v_, sm_scale, block_indices, lens, *a, **kw2):
        captured.append(dict(bi=block_indices.clone(), lens=lens.clone()))
        return torch.zeros_like(q_), torch.zeros(q_.shape[:3])

    def capture(q_, k_, v_, sm_scale, block_indices, lens, *a, **kw2):
        captured.append(dict(bi=block_indices.clone(), lens=lens.clone()))
        return orig(q_, k_, v_, sm_scale, block_indices, lens, *a, **kw2)

    try:
        # pass 1: bf16 inputs, selection only (the kernel call is captured and skipped)
        bsa.attn_fwd_bsa_varlen_triton = skip
        with torch.no_grad():
            _uniform_entry(bsa, case, inp, torch.bfloat16)(q, k, v, **kw)
        sel16 = captured.pop()
        # pass 2: fp32 values (bf16-representable), real kernels, autograd
        bsa.attn_fwd_bsa_varlen_triton = capture
        q32, k32, v32 = (t.float().requires_grad_(True) for t in (q, k, v))
        out = _uniform_entry(bsa, case, inp, torch.float32)(q32, k32, v32, **kw)
        (out * do.float()).sum().backward()
        sel32 = captured.pop()
    finally:
        bsa.attn_fwd_bsa_varlen_triton = orig

    dense16 = chunk_lists_to_dense(sel16["bi"].numpy(), sel16["lens"].numpy(), nk)
    dense32 = chunk_lists_to_dense(sel32["bi"].numpy(), sel32["lens"].numpy(), nk)
    if valid is not None and case.guidance is None:
        assert (dense16 == dense32).all(), "selection differs between bf16 and fp32 passes"
    ar = torch.arange(S, dtype=torch.float64).view(1, 1, S, 1)
    src = []
    for c in (cq, ck):
        n3 = (Tp // c[0], Hp // c[1], Wp // c[2])
        src.append(bsa.rearrange_THW_to_3d_block(ar, *n3, *c, 1).view(-1).long().numpy())
    res = dict(grid=np.array(case.grid), grid_padded=np.array(case.grid_padded),
               chunk_q=np.array(cq), chunk_k=np.array(ck),
               src_idx_q=src[0].astype(np.int32), src_idx_k=src[1].astype(np.int32),
               sel_chunks=dense_to_bits(dense16), sel_chunks_f32=dense_to_bits(dense32))
    o = out.detach()[0].numpy()
    grads = [t.grad[0].numpy() for t in (q32, k32, v32)]
    rng = np.random.default_rng(1234)
    rows = np.sort(rng.choice(S, size=min(S, N_ROWS), replace=False))
    res["rows"] = rows.astype(np.int64)
    res["o"] = o[:, rows]
    res["dq"], res["dk"], res["dv"] = (gr[:, rows] for gr in grads)
    res["sums"] = np.array([np.abs(x).astype(np.float64).sum() for x in [o] + grads])
    if case.guidance is not None:
        res.update(_guidance_parts(bsa, case, inp))
    return res


def run_correction_case(bsa, br, case):
    """bsa_rectified_sparse_attn / bsa_taylor_sparse_attn (bias_rectification.py:
    261-446) under no_grad on CPU (the PyTorch merge, the reference's definition of
    the fused inference kernels), on fp32 values in the 3D-chunk order as the
    correction dispatch of wan_video_dit.py:550-640 passes them.  Stores the chunk
    selection, the reference's R_n, M_n (and is_flat), and the corrected output on
    a fixed subset of rows (chunk order)."""
    from oracle.oracle import dense_to_bits

    inp = make_inputs(case)
    c = case.correction
    Tp, Hp, Wp = case.grid_padded
    S = Tp * Hp * Wp
    D = case.head_dim
    (tq, hq, wq), (tk, hk, wk) = case.chunk_q, case.chunk_k
    cq, ck = tq * hq * wq, tk * hk * wk
    n3q = (Tp // tq, Hp // hq, Wp // wq)
    n3k = (Tp // tk, Hp // hk, Wp // wk)
    q_ro = bsa.rearrange_THW_to_3d_block(inp["q"].float(), *n3q, tq, hq, wq, D)
    k_ro = bsa.rearrange_THW_to_3d_block(inp["k"].float(), *n3k, tk, hk, wk, D)
    v_ro = bsa.rearrange_THW_to_3d_block(inp["v"].float(), *n3k, tk, hk, wk, D)
    valid = inp["valid"]
    vm = None if valid is None else bsa.rearrange_THW_to_3d_block_1d(valid, *n3k, tk, hk, wk)
    sm = 1.0 / D ** 0.5
    mod = None
    if c.get("variance_gamma", 0.0) > 0:
        rho = bsa.compute_channel_variance_density(v_ro, ck, tk, hk, wk, vm)
        mod = (1.0 + c["variance_gamma"] * rho.view(1, 1, 1, -1)).contiguous()
    captured = []
    orig = br.attn_fwd_bsa_varlen_triton

    def capture(q_, k_, v_, sm_scale, block_indices, lens, *a, **kw2):
        captured.append(dict(bi=block_indices.clone(), lens=lens.clone()))
        return orig(q_, k_, v_, sm_scale, block_indices, lens, *a, **kw2)

    kw = dict(chunk_size_q=cq, chunk_size_k=ck, sparsity=case.sparsity,
              cdf_threshold=case.cdf_threshold, sm_scale=sm, kv_valid_mask=vm, score_modifier=mod)
    try:
        br.attn_fwd_bsa_varlen_triton = capture
        with torch.no_grad():
            if c["kind"] == "taylor":
                out = br.bsa_taylor_sparse_attn(q_ro, k_ro, v_ro, alpha_f=c["alpha_f"], **kw)
            else:
                out = br.bsa_rectified_sparse_attn(q_ro, k_ro, v_ro, **kw)
    finally:
        br.attn_fwd_bsa_varlen_triton = orig
    sel = captured.pop()
    nk = S // ck
    dense = chunk_lists_to_dense(sel["bi"].numpy(), sel["lens"].numpy(), nk)
    with torch.no_grad():
        q_cmp, k_cmp = br._pool_qk(q_ro, k_ro, cq, ck, vm, None)
        raw = bsa.cal_score(q_cmp, k_cmp)
        bv = None if vm is None else br._compute_block_valid_mask(vm, ck)
        A = br._masked_softmax_along_last(raw, sm, bv)
        rect = torch.from_numpy(~dense)[None]
        if bv is not None:
            rect = rect & bv.view(1, 1, 1, -1)
        R = (1.0 - (A * rect.to(A.dtype)).sum(dim=-1)).clamp(min=1e-6)
        M = br._masked_var_along_last(A, bv)
    res = dict(sel_chunks_f32=dense_to_bits(dense), R=R[0].numpy(), M=M[0].numpy())
    if c["kind"] == "taylor":
        res["tau"] = np.array(float(torch.quantile(M.float().reshape(-1), c["alpha_f"])))
    o = out[0].numpy()
    rng = np.random.default_rng(1234)
    rows = np.sort(rng.choice(S, size=min(S, 4 * N_ROWS), replace=False))
    res["rows"] = rows.astype(np.int64)
    res["o"] = o[:, rows]
    res["sums"] = np.array([np.abs(o).astype(np.float64).sum()])
    return res


# producer fixtures (inputs.PRODUCER_CASES).  head_dim 128 only: the reference's
# frame / height / width split (head_dim - 2*(head_dim//3), head_dim//3, head_dim//3
# dimensions) covers head_dim/2 frequency pairs only when head_dim//3 is even
# (128 -> 22 + 21 + 21 = 64; 64 -> 11 + 10 + 10 = 31 and rope_apply_head_dim fails)
PRODUCER_CASES = [(n,) + c for n, c in PRODUCER_FIXTURES.items()]


def import_rope_functions(root):
    """precompute_freqs_cis_3d, precompute_freqs_cis and rope_apply_head_dim taken
    unmodified from the reference's wan_video_dit.py (its module imports diffusers,
    absent here, so only these definitions are executed)."""
    import ast

    import einops
    path = f"{root}/hymm/models/modules/wan_video_dit.py"
    tree = ast.parse(open(path).read())
    keep = {"precompute_freqs_cis_3d", "precompute_freqs_cis", "rope_apply_head_dim"}
    mod = ast.Module(body=[n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in keep],
                     type_ignores=[])
    ns = {"torch": torch, "rearrange": einops.rearrange}
    exec(compile(mod, path, "exec"), ns)
    return ns


def run_producer_case(ns, grid, heads, D, seed):
    """The reference's RoPE table for grid (assembled as wan_video_dit.py:1183-1187) and
    q = rope_apply_head_dim(RMSNorm(x)) on seeded bf16 values (torch.nn.RMSNorm, the
    module SelfAttention uses, :226-227)."""
    f, h, w = grid
    fr = ns["precompute_freqs_cis_3d"](D)
    freqs = torch.cat([fr[0][:f].view(f, 1, 1, -1).expand(f, h, w, -1),
                       fr[1][:h].view(1, h, 1, -1).expand(f, h, w, -1),
                       fr[2][:w].view(1, 1, w, -1).expand(f, h, w, -1)], dim=-1).reshape(f * h * w, 1, -1)
    C = heads * D
    x, gamma = make_producer_inputs(grid, heads, D, seed)
    norm = torch.nn.RMSNorm(C, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_(gamma.float())
        normed = norm(x)  # bf16 in -> bf16 out
        y = ns["rope_apply_head_dim"](normed, freqs, D)
    b16 = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return dict(freqs=torch.view_as_real(freqs[:, 0]).numpy(), normed=b16(normed[0]), y=b16(y[0]))


def run_cross_case(bsa, case):
    """flash_attn_bsa_cross (bsa_interface.py:1276-1392) on unpadded inputs.  Stores
    the chunk-level selection of a bf16 and an fp32 pass and the fp32 output / dQ on
    a fixed subset of query rows and dK / dV on a subset of key rows."""
    from oracle.oracle import dense_to_bits

    inp = make_cross_inputs(case)
    q, k, v, do = inp["q"], inp["k"], inp["v"], inp["do"]
    kw = dict(q_grid_size=case.q_shape if case.q_structure == "3d" else None,
              k_grid_size=case.k_shape if case.k_structure == "3d" else None,
              sparsity=case.sparsity, cdf_threshold=case.cdf_threshold,
              chunk_size_q=case.chunk_size_q, chunk_size_k=case.chunk_size_k,
              chunk_3d_shape_q=list(case.chunk_3d_q) if case.chunk_3d_q else None,
              chunk_3d_shape_k=list(case.chunk_3d_k) if case.chunk_3d_k else None)
    captured = []
    orig = bsa.attn_fwd_bsa_varlen_triton

    def skip(q_, k_, v_, sm_scale, block_indices, lens, *a, **kw2):
        captured.append(dict(bi=block_indices.clone(), lens=lens.clone(), nk=k_.shape[2]))
        return torch.zeros_like(q_), torch.zeros(q_.shape[:3])

    def capture(q_, k_, v_, sm_scale, block_indices, lens, *a, **kw2):
        captured.append(dict(bi=block_indices.clone(), lens=lens.clone(), nk=k_.shape[2]))
        return orig(q_, k_, v_, sm_scale, block_indices, lens, *a, **kw2)

    try:
        bsa.attn_fwd_bsa_varlen_triton = skip
        with torch.no_grad():
            bsa.flash_attn_bsa_cross(q, k, v, case.q_structure, case.k_structure, **kw)
        sel16 = captured.pop()
        bsa.attn_fwd_bsa_varlen_triton = capture
        q32, k32, v32 = (t.float().requires_grad_(True) for t in (q, k, v))
        out = bsa.flash_attn_bsa_cross(q32, k32, v32, case.q_structure, case.k_structure, **kw)
        (out * do.float()).sum().backward()
        sel32 = captured.pop()
    finally:
        bsa.attn_fwd_bsa_varlen_triton = orig
    ck = (case.chunk_size_k if case.k_structure == "1d"
          else case.chunk_3d_k[0] * case.chunk_3d_k[1] * case.chunk_3d_k[2])
    nk = sel32["nk"] // ck
    dense16 = chunk_lists_to_dense(sel16["bi"].numpy(), sel16["lens"].numpy(), nk)
    dense32 = chunk_lists_to_dense(sel32["bi"].numpy(), sel32["lens"].numpy(), nk)
    res = dict(sel_chunks=dense_to_bits(dense16), sel_chunks_f32=dense_to_bits(dense32))
    o = out.detach()[0].numpy()
    grads = [t.grad[0].numpy() for t in (q32, k32, v32)]
    rng = np.random.default_rng(1234)
    rows_q = np.sort(rng.choice(case.Sq, size=min(case.Sq, N_ROWS), replace=False))
    rows_k = np.sort(rng.choice(case.Sk, size=min(case.Sk, N_ROWS), replace=False))
    res["rows_q"], res["rows_k"] = rows_q.astype(np.int64), rows_k.astype(np.int64)
    res["o"], res["dq"] = o[:, rows_q], grads[0][:, rows_q]
    res["dk"], res["dv"] = grads[1][:, rows_k], grads[2][:, rows_k]
    res["sums"] = np.array([np.abs(x).astype(np.float64).sum() for x in [o] + grads])
    return res


def main():
    root = os.environ.get("PRISM_REFERENCE")
    if not root:
        sys.exit("set PRISM_REFERENCE to the root of a Prism checkout")
    dba, dbs, bsa = import_reference(root)
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    names = sys.argv[1:] or list(ALL_CASES) + list(CROSS_CASES) + [c[0] for c in PRODUCER_CASES]
    prod = {c[0]: c for c in PRODUCER_CASES}
    for name in names:
        if name in prod:
            _, grid, heads, D, seed = prod[name]
            res = run_producer_case(import_rope_functions(root), grid, heads, D, seed)
            path = os.path.join(HERE, f"{name}.npz")
            np.savez_compressed(path, **res)
            print(f"{name}: rope {grid} x {heads} heads, D={D} -> {path} ({os.path.getsize(path)} B)")
            continue
        path = os.path.join(HERE, f"{name}.npz")
        if name in CROSS_CASES:
            res = run_cross_case(bsa, CROSS_CASES[name])
            np.savez_compressed(path, **res)
            print(f"{name}: cross -> {path} ({os.path.getsize(path)} B)")
            continue
        case = ALL_CASES[name]
        if case.correction is not None:
            res = run_correction_case(bsa, import_bias_rectification(), case)
            np.savez_compressed(path, **res)
            print(f"{name}: {case.correction['kind']} -> {path} ({os.path.getsize(path)} B)")
            continue
        if case.uniform:
            res = run_uniform_case(bsa, case)
            np.savez_compressed(path, **res)
            print(f"{name}: uniform chunks {case.chunk_q}/{case.chunk_k} -> {path} "
                  f"({os.path.getsize(path)} B)")
            continue
        res = run_case(dba, dbs, case)
        np.savez_compressed(path, **res)
        print(f"{name}: shapes {np.bincount(res['shape_ids'], minlength=13).tolist()} "
              f"-> {path} ({os.path.getsize(path)} B)")


if __name__ == "__main__":
    main()
