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
from inputs import CASES, make_inputs  # noqa: E402

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
    return dba, dbs


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


def main():
    root = os.environ.get("PRISM_REFERENCE")
    if not root:
        sys.exit("set PRISM_REFERENCE to the root of a Prism checkout")
    dba, dbs = import_reference(root)
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    names = sys.argv[1:] or list(CASES)
    for name in names:
        case = CASES[name]
        res = run_case(dba, dbs, case)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **res)
        print(f"{name}: shapes {np.bincount(res['shape_ids'], minlength=13).tolist()} "
              f"-> {path} ({os.path.getsize(path)} B)")


if __name__ == "__main__":
    main()
