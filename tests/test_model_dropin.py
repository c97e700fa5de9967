"""The reference's model files through the drop-in.

* CPU (where the reference checkout is present): the unmodified sparse model
  files (src/model_DRUM_kernel_sp.py, src/model_smDRUM_kernel_sp.py,
  src/model_mmDRUM_kernel_sp.py) import under the module alias of the
  integration notes, with flashlog_b200.flashlog_kernel standing in for
  flashlog_kernel.flashlog_kernel: every name they import resolves, and
  every positional .apply call in them binds to the drop-in's forward.
  The GPU box has no reference checkout, so this part runs where it is.
* GPU: the forward of src/model_DRUM_kernel_sp.py:92-201 with the attention
  logits the reference model itself produced (tests/golden/model_drum_sp.npz,
  recorded by make_golden.py --only model from the unmodified model file on
  the reference's own CPU operators), its hops run through the drop-in's
  GPU branch (FlashLogFunctionSparse3DTopKSum.apply, then
  normalize_sparse3d, model lines 150-167 and 195-196) and through its
  CPU-branch call (vectorized_operation_sparse3d_csr_sum_norm, lines
  169-180); channel sum (lines 22-28) and log loss (src/utils.py:36-47) as
  the model file computes them.  The final scores (keys exactly, values at
  rel 1e-5), the loss (rel 1e-5) and the gradient of every channel's logits
  (rel 1e-5 with an absolute floor of 1e-6 x the largest magnitude, as the
  softmax backward subtracts terms) match the reference model's run.
"""
import ast
import inspect
import os
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")

MODEL_FILES = ("model_DRUM_kernel_sp.py", "model_smDRUM_kernel_sp.py", "model_mmDRUM_kernel_sp.py")


def _reference_src():
    from oracle.build import reference_root
    root = reference_root()
    src = os.path.join(root, "src") if root else None
    return src if src and all(os.path.exists(os.path.join(src, f)) for f in MODEL_FILES) else None


def test_reference_model_files_bind_to_the_dropin():
    src = _reference_src()
    if src is None:
        pytest.skip("the reference checkout is not present (it is not shipped to the GPU box)")
    import flashlog_b200 as pkg
    import flashlog_b200.flashlog_kernel as fk
    saved = {k: sys.modules.get(k) for k in ("flashlog_kernel", "flashlog_kernel.flashlog_kernel")}
    sys.modules["flashlog_kernel"] = pkg
    sys.modules["flashlog_kernel.flashlog_kernel"] = fk
    sys.path.insert(0, src)
    try:
        import importlib
        for fname in MODEL_FILES:
            mod = importlib.import_module(fname[:-3])
            tree = ast.parse(open(os.path.join(src, fname)).read())
            names = [a.name for node in ast.walk(tree) if isinstance(node, ast.ImportFrom)
                     and node.module == "flashlog_kernel.flashlog_kernel" for a in node.names]
            assert names, fname
            for nm in names:
                assert getattr(mod, nm) is getattr(fk, nm), (fname, nm)
            for node in ast.walk(tree):
                if (isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute) and node.func.attr == "apply"
                        and isinstance(node.func.value, ast.Name) and hasattr(fk, node.func.value.id)):
                    fwd = getattr(fk, node.func.value.id).forward
                    n_params = len(inspect.signature(fwd).parameters) - 1  # ctx
                    required = sum(1 for p in list(inspect.signature(fwd).parameters.values())[1:]
                                   if p.default is inspect.Parameter.empty)
                    assert required <= len(node.args) <= n_params, (fname, node.func.value.id, len(node.args))
    finally:
        sys.path.remove(src)
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
        for fname in MODEL_FILES:
            sys.modules.pop(fname[:-3], None)


def _sum_sp_3d(s):
    # src/model_DRUM_kernel_sp.py:22-28
    s = s.coalesce()
    idx = s.indices()
    B, L, E = s.shape
    return torch.sparse_coo_tensor(torch.stack([idx[0], idx[2]]), s.values(), [B, E]).coalesce()


def _log_loss(p_score, label, E, tau_2, thr=1e-7):
    # src/utils.py:36-47
    i = torch.stack([torch.arange(label.shape[0], device=label.device), label.long()])
    one_hot = torch.sparse_coo_tensor(i, torch.ones_like(label).float(), (label.shape[0], E))
    logits = torch.sparse.sum(p_score * one_hot, dim=-1).to_dense()
    return -torch.mean(torch.log(torch.maximum(logits / tau_2, torch.ones_like(logits) * thr)), dim=-1)


@pytest.mark.gpu
@pytest.mark.parametrize("branch", ["gpu", "cpu_call"])
def test_reference_model_forward_through_the_dropin(golden, branch):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import flashlog_b200.flashlog_kernel as fk
    from flashlog_b200.synthetic import CONFIGS, load_or_generate
    d = golden("model_drum_sp.npz")
    cfg = CONFIGS[1]
    train, _, _ = load_or_generate(cfg)
    E, R = cfg.entities, cfg.relations
    dev = torch.device("cuda")
    tt = torch.from_numpy(train).to(dev)
    csr = fk.build_csr_structure(tt[:, 0], tt[:, 2], tt[:, 1], E)
    (ori_row_ptr, ori_col_ind, ori_r_ind, order_ori, inv_row_ptr, inv_col_ind, inv_r_ind, order_inv,
     ori_gptr, ori_grel, ori_gstart, ori_gcount, inv_gptr, inv_grel, inv_gstart, inv_gcount) = csr
    mask = torch.ones(train.shape[0], dtype=torch.bool, device=dev)
    mask[torch.from_numpy(d["hidden"]).to(dev)] = False
    c1, c2, tau_1, tau_2 = int(d["c1"]), int(d["c2"]), float(d["tau_1"]), float(d["tau_2"])
    logits = [torch.from_numpy(d[f"logits{l}"]).to(dev).requires_grad_(True) for l in range(3)]
    w_all = torch.stack(logits, dim=2)  # [B, T, L, n]
    x = torch.from_numpy(d["heads"]).to(dev)
    B, T, L = x.shape[0], w_all.shape[1], w_all.shape[2]
    r_size = R
    sp_batch = torch.arange(B, device=dev).repeat_interleave(L)
    sp_level = torch.arange(L, device=dev).repeat(B)
    sp_entity = x.long().repeat_interleave(L)
    sp_value = torch.ones(B * L, device=dev)
    state = torch.sparse_coo_tensor(torch.stack([sp_batch, sp_level, sp_entity]), sp_value, [B, L, E]).coalesce()
    for t in range(T):
        w_t = torch.softmax(w_all[:, t, :, :] / tau_1, dim=-1)
        if branch == "gpu":
            s = fk.FlashLogFunctionSparse3DTopKSum.apply(
                sp_batch, sp_level, sp_entity, sp_value, w_t,
                ori_row_ptr, ori_col_ind, ori_r_ind, order_ori,
                inv_row_ptr, inv_col_ind, inv_r_ind, order_inv,
                ori_gptr, ori_grel, ori_gstart, ori_gcount, inv_gptr, inv_grel, inv_gstart, inv_gcount,
                mask, None, B, L, E, r_size, False, c2 // 2, False, c1, torch.is_grad_enabled())
            s = fk.normalize_sparse3d(s)
        else:
            state_sp = torch.sparse_coo_tensor(torch.stack([sp_batch, sp_level, sp_entity]), sp_value,
                                               [B, L, E]).coalesce()
            s = fk.vectorized_operation_sparse3d_csr_sum_norm(state_sp, w_t, csr, mask, r_size, weight=None,
                                                              use_topk=True, topk_edges=c2 // 2, topk_nodes=c1)
        s_c = s if s.is_coalesced() else s.coalesce()
        sp_batch, sp_level, sp_entity = s_c.indices()[0], s_c.indices()[1], s_c.indices()[2]
        sp_value = s_c.values()
        state = s
    final = _sum_sp_3d(state)
    loss = _log_loss(final, torch.from_numpy(d["tails"]).to(dev), E, tau_2)
    loss.backward()
    fi = final.indices().cpu().numpy()
    assert np.array_equal(fi[0] * E + fi[1], d["final_key"])
    np.testing.assert_allclose(final.values().detach().cpu().numpy(), d["final_val"], rtol=1e-5, atol=0)
    assert float(loss) == pytest.approx(float(d["loss"]), rel=1e-5)
    for l in range(3):
        want = d[f"grad{l}"]
        np.testing.assert_allclose(logits[l].grad.cpu().numpy(), want, rtol=1e-5,
                                   atol=1e-6 * float(np.abs(want).max()))
