"""Attributors against brute-force oracles on a tiny MLP (CPU).

Per-sample gradients come from autograd one sample at a time; the oracles
build every quantity explicitly (dense Kronecker inverses, eigenbases, products
of Fisher factors), independent of the package's fast paths.
"""

from __future__ import annotations

import warnings

import pytest
import torch

from dattri_llm_b200.attribution import (
    AdamWInfluenceAttributor,
    AttributionArguments,
    AttributionScore,
    DVEmbAttributor,
    EKFACAttributor,
    KFACAttributor,
    LESSAttributor,
    TracInAttributor,
)
from dattri_llm_b200.gradient import ops
from dattri_llm_b200.gradient.hooks import HookManagerConfig
from dattri_llm_b200.gradient.storage_manager import GradientStorageManager
from dattri_llm_b200.task import AttributionTask
from tests import tiny

warnings.filterwarnings("ignore", category=UserWarning)


def _args(path, **kw) -> AttributionArguments:
    return AttributionArguments(output_dir=str(path), use_cpu=True, **kw)


def _matrix(res: AttributionScore, train_ids, test_ids) -> torch.Tensor:
    return res.query(train_ids, test_ids, trajectory="agnostic")


@pytest.fixture
def single_step(tmp_path):
    model = tiny.make_model()
    xtr, ytr, xte, yte = tiny.make_data()
    sd = tiny.checkpoints(model, 1)
    tiny.collect_to_disk(model, sd, xtr, ytr, tmp_path / "tr")
    tiny.collect_to_disk(model, sd, xte, yte, tmp_path / "te")
    model.load_state_dict(sd[0])
    return {"tr": str(tmp_path / "tr"), "te": str(tmp_path / "te"), "model": model,
            "trh": tiny.hashes(xtr, ytr), "teh": tiny.hashes(xte, yte),
            "G": tiny.per_sample_grads(model, xtr, ytr), "T": tiny.per_sample_grads(model, xte, yte),
            "ftr": tiny.factors(model, xtr, ytr), "fte": tiny.factors(model, xte, yte)}


class TestTracIn:
    @pytest.mark.parametrize("loop_over_test", [False, True])
    def test_gradient_dot(self, single_step, tmp_path, loop_over_test):
        d = single_step
        res = TracInAttributor(_args(tmp_path / "o")).attribute_from_cache(d["tr"], d["te"],
                                                                            loop_over_test=loop_over_test)
        got = _matrix(res, d["trh"], d["teh"])
        torch.testing.assert_close(got, d["G"] @ d["T"].T, rtol=1e-4, atol=1e-4)

    def test_checkpoints_sum(self, tmp_path):
        model = tiny.make_model()
        xtr, ytr, xte, yte = tiny.make_data()
        cks = tiny.checkpoints(model, 2)
        tiny.collect_to_disk(model, cks, xtr, ytr, tmp_path / "tr")
        tiny.collect_to_disk(model, cks[:1], xte, yte, tmp_path / "te")
        model.load_state_dict(cks[0])
        q = tiny.per_sample_grads(model, xte, yte)
        want = torch.zeros(tiny.N_TRAIN, tiny.N_TEST)
        for sd in cks:
            model.load_state_dict(sd)
            want += tiny.per_sample_grads(model, xtr, ytr) @ q.T
        res = TracInAttributor(_args(tmp_path / "o")).attribute_from_cache(str(tmp_path / "tr"), str(tmp_path / "te"))
        assert sorted(set(res.row_steps)) == [0, 1]
        torch.testing.assert_close(_matrix(res, tiny.hashes(xtr, ytr), tiny.hashes(xte, yte)), want,
                                   rtol=1e-4, atol=1e-4)

    def test_normalized(self, single_step, tmp_path):
        d = single_step
        res = TracInAttributor(_args(tmp_path / "o")).attribute_from_cache(d["tr"], d["te"], normalized_grad=True)
        nrm = torch.nn.functional.normalize
        torch.testing.assert_close(_matrix(res, d["trh"], d["teh"]), nrm(d["G"], dim=1) @ nrm(d["T"], dim=1).T,
                                   rtol=1e-4, atol=1e-5)

    def test_score_roundtrip_and_topk(self, single_step, tmp_path):
        d = single_step
        res = TracInAttributor(_args(tmp_path / "o")).attribute_from_cache(d["tr"], d["te"])
        back = AttributionScore.load(res.save(tmp_path / "saved"))
        torch.testing.assert_close(back.scores, res.scores)
        assert back.row_train_ids == res.row_train_ids and back.test_ids == res.test_ids
        vals, ids = res.topk(3)
        m = _matrix(res, res.train_ids, res.test_ids)
        for j in range(m.shape[1]):
            torch.testing.assert_close(vals[:, j] if vals.shape[0] == 3 else vals[j], m[:, j].topk(3).values)


def _kfac_oracle(ftr, fte, damping):
    out = 0
    for n in tiny.LAYERS:
        a, g = ftr[n]
        at, gt = fte[n]
        n_s = a.shape[0]
        ai = torch.linalg.inv(a.T @ a / n_s + damping * torch.eye(a.shape[1]))
        gi = torch.linalg.inv(g.T @ g / n_s + damping * torch.eye(g.shape[1]))
        dtr = torch.einsum("no,ni->noi", g, a)
        dte = torch.einsum("mo,mi->moi", gt, at)
        out = out + torch.einsum("noi,moi->nm", dtr, gi @ dte @ ai)
    return out


def _ekfac_oracle(ftr, fte, damping):
    out = 0
    for n in tiny.LAYERS:
        a, g = ftr[n]
        at, gt = fte[n]
        n_s = a.shape[0]
        _, ua = torch.linalg.eigh((a.T @ a / n_s).double())
        _, ug = torch.linalg.eigh((g.T @ g / n_s).double())
        ua, ug = ua.float(), ug.float()
        rtr = torch.einsum("op,no,ni,iq->npq", ug, g, a, ua)
        rte = torch.einsum("op,mo,mi,iq->mpq", ug, gt, at, ua)
        lam = (rtr * rtr).mean(0)
        out = out + torch.einsum("npq,mpq->nm", rtr / (lam + damping), rte)
    return out


class TestKronecker:
    @pytest.mark.parametrize("damping", [1e-2, 1.0])
    def test_kfac(self, single_step, tmp_path, damping):
        d = single_step
        res = KFACAttributor(_args(tmp_path / "o")).attribute_from_cache(d["tr"], d["te"], damping=damping)
        want = _kfac_oracle(d["ftr"], d["fte"], damping)
        torch.testing.assert_close(_matrix(res, d["trh"], d["teh"]), want, rtol=2e-3, atol=2e-3 * want.abs().max())

    @pytest.mark.parametrize("damping", [1e-2, 1.0])
    def test_ekfac(self, single_step, tmp_path, damping):
        d = single_step
        res = EKFACAttributor(_args(tmp_path / "o")).attribute_from_cache(d["tr"], d["te"], damping=damping)
        want = _ekfac_oracle(d["ftr"], d["fte"], damping)
        torch.testing.assert_close(_matrix(res, d["trh"], d["teh"]), want, rtol=2e-3, atol=2e-3 * want.abs().max())

    @pytest.mark.parametrize("cls", [KFACAttributor, EKFACAttributor])
    def test_heavy_damping_is_gradient_dot(self, single_step, tmp_path, cls):
        d = single_step
        lam = 1e6
        res = cls(_args(tmp_path / "o")).attribute_from_cache(d["tr"], d["te"], damping=lam)
        want = d["G"] @ d["T"].T
        scale = lam if cls is EKFACAttributor else lam * lam
        torch.testing.assert_close(_matrix(res, d["trh"], d["teh"]) * scale, want, rtol=1e-3, atol=1e-3)

    def test_fisher_dir_reuse(self, single_step, tmp_path):
        d = single_step
        first = KFACAttributor(_args(tmp_path / "a"))
        res1 = first.attribute_from_cache(d["tr"], d["te"], damping=0.1, fisher_dir=str(tmp_path / "fisher"))
        assert (tmp_path / "fisher" / "fisher_factors.pt").exists()
        res2 = KFACAttributor(_args(tmp_path / "b")).attribute_from_cache(d["tr"], d["te"], damping=0.1,
                                                                          fisher_dir=str(tmp_path / "fisher"))
        torch.testing.assert_close(res1.scores, res2.scores)


def _multi_step(tmp_path, n_ck=3):
    """Steps ``2c`` / ``2c+1``: the two halves of the train set at checkpoint ``c``."""
    model = tiny.make_model()
    xtr, ytr, xte, yte = tiny.make_data()
    cks = tiny.checkpoints(model, n_ck)
    tiny.collect_to_disk(model, cks, xtr, ytr, tmp_path / "tr", batch_size=4)
    tiny.collect_to_disk(model, cks[-1:], xte, yte, tmp_path / "te")
    trh = tiny.hashes(xtr, ytr)
    steps = {}
    for c, sd in enumerate(cks):
        model.load_state_dict(sd)
        g = tiny.per_sample_grads(model, xtr, ytr)
        steps[2 * c], steps[2 * c + 1] = (g[:4], trh[:4]), (g[4:], trh[4:])
    model.load_state_dict(cks[-1])
    return {"tr": str(tmp_path / "tr"), "te": str(tmp_path / "te"), "steps": steps,
            "T": tiny.per_sample_grads(model, xte, yte), "teh": tiny.hashes(xte, yte)}


def _dvemb_oracle(steps, test, lr, mode):
    d = test.shape[1]
    widths = (tiny.IN * tiny.HID, tiny.HID * tiny.OUT)
    out = {}
    for t in steps:
        prod = torch.eye(d, dtype=torch.float64)
        for s in sorted(steps):
            if s <= t:
                continue
            g = steps[s][0].double()
            if mode == "full":
                h = g.T @ g
            else:
                h = torch.zeros(d, d, dtype=torch.float64)
                o = 0
                for w in widths:
                    h[o:o + w, o:o + w] = g[:, o:o + w].T @ g[:, o:o + w]
                    o += w
            prod = prod @ (torch.eye(d, dtype=torch.float64) - lr * g.shape[0] * h)
        out[t] = (lr * steps[t][0].double() @ prod @ test.double().T).float()
    return out


class TestDVEmb:
    @pytest.mark.parametrize("mode", ["full", "diagonal"])
    @pytest.mark.parametrize("prop", ["train", "test", "test-loop"])
    def test_matches_fisher_product(self, tmp_path, mode, prop):
        d = _multi_step(tmp_path)
        lr = 0.05
        res = DVEmbAttributor(_args(tmp_path / "o")).attribute_from_cache(
            d["tr"], d["te"], learning_rate=lr, hessian_mode=mode, propagation=prop.split("-")[0],
            loop_over_test=prop.endswith("loop"))
        want = _dvemb_oracle(d["steps"], d["T"], lr, mode)
        cols = [res.test_index[h] for h in d["teh"]]
        for t, (_g, ids) in d["steps"].items():
            row_ids, m = res.step_matrix(t)
            got = m[[row_ids.index(h) for h in ids]][:, cols]
            torch.testing.assert_close(got, want[t], rtol=1e-3, atol=1e-3 * want[t].abs().max())

    def test_selected_steps_and_dvemb_dir(self, tmp_path):
        d = _multi_step(tmp_path)
        res = DVEmbAttributor(_args(tmp_path / "o")).attribute_from_cache(
            d["tr"], d["te"], learning_rate=0.05, selected_training_steps=[1, 3], dvemb_dir=str(tmp_path / "emb"))
        assert sorted(set(res.row_steps)) == [1, 3]
        again = TracInAttributor(_args(tmp_path / "t")).attribute_from_cache(str(tmp_path / "emb"), d["te"])
        for t in (1, 3):
            ids, m = res.step_matrix(t)
            ids2, m2 = again.step_matrix(t)
            torch.testing.assert_close(m2[[ids2.index(h) for h in ids]], m, rtol=1e-4, atol=1e-5)

    def test_rejects_bad_options(self, tmp_path):
        d = _multi_step(tmp_path, 1)
        a = DVEmbAttributor(_args(tmp_path / "o"))
        with pytest.raises(ValueError):
            a.attribute_from_cache(d["tr"], d["te"], propagation="train", loop_over_test=True)
        with pytest.raises(ValueError):
            a.attribute_from_cache(d["tr"], d["te"], hessian_mode="kfac")
        with pytest.raises(ValueError):
            a.attribute_from_cache(d["tr"], d["te"], propagation="test", dvemb_dir=str(tmp_path / "x"))
        with pytest.raises(ValueError):
            a.attribute_from_cache(d["tr"], d["te"], learning_rate={0: 0.1, 5: 0.1})


def _live(tmp_path, cls, name, **kw):
    model = tiny.make_model()
    xtr, ytr, xte, yte = tiny.make_data()
    sd0 = {k: v.clone() for k, v in model.state_dict().items()}
    task = AttributionTask(tiny.sq_loss, model, checkpoints=[sd0])
    args = _args(tmp_path / name, per_device_train_batch_size=4, per_device_eval_batch_size=4, learning_rate=0.05,
                 max_grad_norm=None, lr_scheduler_type="constant", **kw)
    return cls(args, task=task), tiny.as_dataset(xtr, ytr), tiny.as_dataset(xte, yte), task


class TestAdamWInfluence:
    def test_train_and_test_propagation_agree(self, tmp_path):
        attr, train, test, _ = _live(tmp_path, AdamWInfluenceAttributor, "o", adam_epsilon=0.1)
        hc = HookManagerConfig(linear_io=[r"mlp\."])
        attr.cache(train, test, hook_config=hc)
        root = tmp_path / "o"
        r_train = attr.attribute_from_cache(str(root / "train_grads"), str(root / "test_grads"), propagation="train")
        r_test = attr.attribute_from_cache(str(root / "train_grads"), str(root / "test_grads"), propagation="test")
        r_loop = attr.attribute_from_cache(str(root / "train_grads"), str(root / "test_grads"), propagation="test",
                                           loop_over_test=True)
        assert r_train.row_train_ids == r_test.row_train_ids
        torch.testing.assert_close(r_test.scores, r_train.scores, rtol=1e-3, atol=1e-5)
        torch.testing.assert_close(r_loop.scores, r_train.scores, rtol=1e-3, atol=1e-5)

    def test_last_step_is_adam_push(self, tmp_path):
        """At the final step nothing propagates: the score is ``-g_q . theta_dot(z)``."""
        attr, train, test, task = _live(tmp_path, AdamWInfluenceAttributor, "o", adam_epsilon=0.1)
        hc = HookManagerConfig(linear_io=[r"mlp\."])
        attr.cache(train, test, hook_config=hc)
        root = tmp_path / "o"
        dyn = torch.load(root / "train_grads" / "adamw_dynamics.pt", weights_only=False)
        last = max(dyn)
        res = attr.attribute_from_cache(str(root / "train_grads"), str(root / "test_grads"),
                                        selected_training_steps=[last])
        e = dyn[last]
        b1, b2 = e["betas"]
        t = int(e["step"])
        cat = lambda side, i: torch.cat([e[side][n][i].reshape(-1) for n in sorted(e[side])])  # noqa: E731
        m_post, v_post, m_pre = cat("post", 0), cat("post", 1), cat("pre", 0)
        g_t = (m_post - b1 * m_pre) / (1 - b1)
        root_v = (v_post / (1 - b2**t)).sqrt()
        dd = 1 / (root_v + e["eps"])
        ss = (m_post / (1 - b1**t)) / (2 * root_v * (root_v + e["eps"]) ** 2)
        ids, m = res.step_matrix(last)

        def rows(path, step):
            store = GradientStorageManager(str(path))
            out, hs = [], []
            for f, by_step in store.iter_steps(step):
                recs = store.load_records(f)
                for i in by_step[step]:
                    g = recs[i].gradient
                    dense = [ops.materialize(g.data[n], g.layer_types[n]) for n in sorted(g.data)]
                    out.append(torch.cat([v.reshape(v.shape[0], -1).float() for v in dense], 1))
                    hs.extend(recs[i].input_hash if isinstance(recs[i].input_hash, list) else [recs[i].input_hash])
            return torch.cat(out), hs

        gz, zh = rows(root / "train_grads", last)
        gq, qh = rows(root / "test_grads", min(GradientStorageManager(str(root / "test_grads")).available_steps()))
        m_dot = -(1 - b1) * gz
        v_dot = -2 * (1 - b2) * g_t * gz
        theta_dot = -e["lr"] * (dd * m_dot / (1 - b1**t) - ss * v_dot / (1 - b2**t))
        want = -(theta_dot @ gq.T)
        got = m[[ids.index(h) for h in zh]][:, [res.test_index[h] for h in qh]]
        torch.testing.assert_close(got, want, rtol=1e-3, atol=1e-5)


class TestLESS:
    def test_frozen_form_cosine(self, tmp_path):
        model = tiny.make_model()
        xtr, ytr, xte, yte = tiny.make_data()
        cks = tiny.checkpoints(model, 2)
        optimizers, dirs = [], []
        for c, sd in enumerate(cks):
            model.load_state_dict(sd)
            opt = torch.optim.Adam(model.parameters(), lr=1e-3, betas=(0.9, 0.99), eps=1e-6)
            for k in range(2 + c):
                model.zero_grad()
                tiny.sq_loss(model, {"x": xtr[k:k + 3] * (1 + c), "y": ytr[k:k + 3]}).backward()
                opt.step()
            model.load_state_dict(sd)
            optimizers.append(opt)
        want = torch.zeros(tiny.N_TRAIN, tiny.N_TEST)
        for c, sd in enumerate(cks):
            model.load_state_dict(sd)
            g = tiny.per_sample_grads(model, xtr, ytr)
            q = tiny.per_sample_grads(model, xte, yte)
            st = optimizers[c].state
            m0 = torch.cat([st[dict(model.named_parameters())[n]]["exp_avg"].reshape(-1) for n in tiny.WEIGHTS])
            v0 = torch.cat([st[dict(model.named_parameters())[n]]["exp_avg_sq"].reshape(-1) for n in tiny.WEIGHTS])
            step = int(st[model.mlp.fc1.weight]["step"]) + 1
            m = 0.9 * m0 + 0.1 * g
            v = 0.99 * v0 + 0.01 * g * g
            dvec = (m / (1 - 0.9**step)) / ((v / (1 - 0.99**step)).sqrt() + 1e-6)
            dirs.append(dvec)
            want += torch.nn.functional.normalize(dvec, dim=1) @ torch.nn.functional.normalize(q, dim=1).T
        sd0 = {k: v.clone() for k, v in cks[0].items()}
        task = AttributionTask(tiny.sq_loss, model, checkpoints=[sd0, cks[1]])
        args = _args(tmp_path / "o", per_device_train_batch_size=4, per_device_eval_batch_size=4)
        res = LESSAttributor(args, task=task, optimizers=optimizers).attribute(
            tiny.as_dataset(xtr, ytr), tiny.as_dataset(xte, yte), hook_config=HookManagerConfig(linear_io=[r"mlp\."]))
        got = _matrix(res, tiny.hashes(xtr, ytr), tiny.hashes(xte, yte))
        torch.testing.assert_close(got, want, rtol=1e-3, atol=1e-4)


class TestTrajectoryLive:
    @pytest.mark.parametrize("residency", ["disk", "memory"])
    def test_dvemb_live_matches_cached(self, tmp_path, residency):
        attr, train, test, _ = _live(tmp_path, DVEmbAttributor, "o", optim="sgd")
        hc = HookManagerConfig(linear_io=[r"mlp\."])
        live = attr.attribute(train, test, hook_config=hc, learning_rate=0.05, gradient_cache_residency=residency)
        assert live.scores.shape == (tiny.N_TRAIN, tiny.N_TEST)
        assert sorted(set(live.row_steps)) == [0, 1]
        attr2, train, test, _ = _live(tmp_path, DVEmbAttributor, "p", optim="sgd")
        ((trd, ted),) = attr2.cache(train, test, hook_config=hc)
        cached = attr2.attribute_from_cache(trd, ted, learning_rate=0.05)
        torch.testing.assert_close(live.scores, cached.scores, rtol=1e-4, atol=1e-6)

    def test_trajectory_reloads_checkpoint_afterwards(self, tmp_path):
        attr, train, test, task = _live(tmp_path, DVEmbAttributor, "o", optim="sgd")
        before = {k: v.clone() for k, v in task.get_model().state_dict().items()}
        attr.cache(train, test, hook_config=HookManagerConfig(linear_io=[r"mlp\."]))
        assert task.current_checkpoint_idx is None
        after = task.load_checkpoint(0).state_dict()
        for k, v in before.items():
            torch.testing.assert_close(after[k], v)


def _same_scores(a, b) -> None:
    """Equal per-step score rows, aligned by train id and test id."""
    assert sorted(set(a.row_steps)) == sorted(set(b.row_steps))
    for step in set(a.row_steps):
        ids_a, ma = a.step_matrix(step)
        ids_b, mb = b.step_matrix(step)
        assert sorted(ids_a) == sorted(ids_b)
        ca = [a.test_index[h] for h in a.test_ids]
        cb = [b.test_index[h] for h in a.test_ids]
        mb = mb[[ids_b.index(h) for h in ids_a]]
        torch.testing.assert_close(mb[:, cb], ma[:, ca], rtol=1e-4, atol=1e-6)


class TestRecompute:
    def test_snapshot_replay_equals_stored_trajectory(self, tmp_path):
        """``recompute_gradients=True`` stores parameters + batches and replays the
        gradients at attribution time; the scores equal the stored-gradient run."""
        hc = HookManagerConfig(linear_io=[r"mlp\."])
        stored, train, test, _ = _live(tmp_path, DVEmbAttributor, "stored", optim="sgd")
        a = stored.attribute(train, test, hook_config=hc, learning_rate=0.05)
        replay, train, test, _ = _live(tmp_path, DVEmbAttributor, "replay", optim="sgd", recompute_gradients=True)
        b = replay.attribute(train, test, hook_config=hc, learning_rate=0.05)
        _same_scores(a, b)

    def test_adamw_replay_equals_stored(self, tmp_path):
        hc = HookManagerConfig(linear_io=[r"mlp\."])
        stored, train, test, _ = _live(tmp_path, AdamWInfluenceAttributor, "s", adam_epsilon=0.1)
        a = stored.attribute(train, test, hook_config=hc)
        replay, train, test, _ = _live(tmp_path, AdamWInfluenceAttributor, "r", adam_epsilon=0.1,
                                       recompute_gradients=True)
        b = replay.attribute(train, test, hook_config=hc)
        _same_scores(a, b)


class TestLiveAttribute:
    @pytest.mark.parametrize("residency", ["disk", "memory"])
    def test_tracin_live_equals_cached(self, tmp_path, residency):
        model = tiny.make_model()
        xtr, ytr, xte, yte = tiny.make_data()
        task = AttributionTask(tiny.sq_loss, model, checkpoints=[{k: v.clone() for k, v in model.state_dict().items()}])
        args = _args(tmp_path / "o", per_device_train_batch_size=4, per_device_eval_batch_size=4)
        hc = HookManagerConfig(linear_io=[r"mlp\."])
        live = TracInAttributor(args, task=task).attribute(tiny.as_dataset(xtr, ytr), tiny.as_dataset(xte, yte),
                                                           hook_config=hc, gradient_cache_residency=residency)
        model.load_state_dict(task.checkpoints[0])
        want = tiny.per_sample_grads(model, xtr, ytr) @ tiny.per_sample_grads(model, xte, yte).T
        torch.testing.assert_close(_matrix(live, tiny.hashes(xtr, ytr), tiny.hashes(xte, yte)), want,
                                   rtol=1e-4, atol=1e-4)

    def test_token_granularity_sums_to_instance(self, tmp_path):
        """Per-token scores of a train sample sum to its instance score (TracIn)."""
        torch.manual_seed(0)
        model = torch.nn.Sequential()
        model.add_module("fc", torch.nn.Linear(6, 3))
        x = torch.randn(4, 5, 6)
        data = [{"x": x[i]} for i in range(4)]

        def loss_fn(m, b):
            return m(b["x"]).pow(2).sum()

        task = AttributionTask(loss_fn, model)
        args = _args(tmp_path / "o", per_device_train_batch_size=2, per_device_eval_batch_size=2)
        hc = HookManagerConfig(linear_io=[r"^fc$"])
        inst = TracInAttributor(args, task=task).attribute(data, data[:2], hook_config=hc)
        tok = TracInAttributor(_args(tmp_path / "t", per_device_train_batch_size=2, per_device_eval_batch_size=2),
                               task=task).attribute(data, data[:2], hook_config=hc, attribution_granularity="token")
        for h in inst.train_ids:
            for step in set(inst.row_steps):
                _pos, per_tok = tok.token_scores(h, step)
                torch.testing.assert_close(per_tok.sum(0), inst.trajectory_agnostic(h), rtol=1e-4, atol=1e-5)
