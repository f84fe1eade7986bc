import os

import torch

from psrl_b200.config import load_config
from psrl_b200.models import PRESETS, build_model
from psrl_b200.models.hf_io import from_hf_state_dict, load_hf_into, save_hf, to_hf_state_dict


def test_hf_roundtrip_dense_and_moe(tmp_path):
    for preset in ("tiny", "tiny-moe"):
        a = PRESETS[preset]
        m = build_model(a, "cpu", torch.float32, seed=3)
        sd = {k: v for k, v in m.state_dict().items()}
        hf = to_hf_state_dict(sd, a)
        assert "model.layers.0.self_attn.q_proj.weight" in hf
        back = from_hf_state_dict(hf, a)
        for k, v in sd.items():
            assert torch.equal(back[k], v), k
        d = str(tmp_path / preset)
        save_hf(m, d)
        m2 = build_model(a, "cpu", torch.float32, seed=9)
        load_hf_into(m2, d)
        for (k, v), (_, w) in zip(m.named_parameters(), m2.named_parameters()):
            assert torch.equal(v, w), k


def test_trainer_checkpoint_resume(tmp_path):
    from psrl_b200.trainer import RLTrainer
    root = str(tmp_path / "ckpt")
    cfg = load_config(preset="cpu_tiny_grpo", overrides=[f"trainer.default_local_dir={root}",
                                                         "psrl.checkpoint.use_dcp_save=false"])
    t = RLTrainer(cfg)
    t.step()
    t.step()
    t.save_checkpoint()
    assert open(os.path.join(root, "latest_checkpointed_iteration.txt")).read() == "2"
    ref = {k: v.clone() for k, v in t.actor.model.named_parameters()}
    cursor = t.data.cursor
    cfg2 = load_config(preset="cpu_tiny_grpo", overrides=[f"trainer.default_local_dir={root}",
                                                          "psrl.checkpoint.use_dcp_save=false",
                                                          "trainer.resume_mode=auto"])
    t2 = RLTrainer(cfg2, seed=99)
    step = t2.resume()
    assert step == 2 and t2.global_step == 2
    assert t2.data.cursor == cursor
    assert t2.ps.get_ps_model_version() == 2
    for k, v in t2.actor.model.named_parameters():
        assert torch.equal(v, ref[k]), k
    assert t2.actor.dp.step_count == t.actor.dp.step_count
    m = t2.step()                  # continues from buffer 2
    assert m["step"] == 2


def test_adaptive_kl_coefficient_survives_resume(tmp_path):
    from psrl_b200.trainer import RLTrainer
    root = str(tmp_path / "ckpt")
    ov = [f"trainer.default_local_dir={root}", "psrl.checkpoint.use_dcp_save=false",
          "algorithm.use_kl_in_reward=true", "algorithm.kl_ctrl.type=adaptive", "rollout.max_response_length=12"]
    t = RLTrainer(load_config(preset="cpu_tiny_grpo", overrides=ov))
    t.step()
    t.save_checkpoint()
    t.stop_rollout()
    coef = t.kl_ctrl.value
    assert coef != 0.001
    t2 = RLTrainer(load_config(preset="cpu_tiny_grpo", overrides=ov + ["trainer.resume_mode=auto"]), seed=7)
    assert t2.resume() == 1
    assert t2.kl_ctrl.value == coef
