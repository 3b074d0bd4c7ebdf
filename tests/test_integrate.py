"""install_refiner on a stand-in MoGeModel (CPU): the hook binds to the refine loop's two methods, reads the model's
own QAT refiner, and refuses what the B200 plan does not run (no CPU path, no non-QAT refiner, other layouts)."""
import pytest
import torch

from stub_moge import stub_model


def test_install_binds_the_loop_methods_and_uninstall_restores_them():
    from promptmoge_b200.integrate import install_refiner, uninstall_refiner
    m = stub_model("B")
    hook = install_refiner(m)
    assert m._refine_logz == hook.refine_logz and m._lidar_in_affine_frame == hook.lidar_in_affine_frame
    assert install_refiner(m) is hook                       # idempotent
    assert hook.geo == dict(channels=[32, 64, 128, 256], enc_channels=1024, prompt_channels=2, encoder_downsample=8)
    assert len(hook.clips) == 25 and "down_stages.0.0.conv1" in hook.clips
    assert hook.weights["down_stages.0.0.conv1.weight"].shape == (32, 3, 3, 3, 32)
    uninstall_refiner(m)
    with pytest.raises(AssertionError, match="not installed"):
        m._refine_logz(None, None)


def test_hook_has_no_cpu_path():
    from promptmoge_b200.integrate import install_refiner
    m = stub_model("B")
    install_refiner(m)
    pc = torch.zeros(1, 240, 320, 3)
    enc = torch.zeros(1, 1024, 30, 40, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        m._refine_logz(pc, enc, prompt_feats=torch.zeros(240 * 320, 2))
    with pytest.raises(RuntimeError, match="CUDA"):
        m._lidar_in_affine_frame(pc[..., 2], torch.ones(1, 1, 192, 256), torch.ones(1, 1, 192, 256))


def test_refuses_refiners_the_plan_does_not_run():
    from promptmoge_b200.integrate import install_refiner
    with pytest.raises(ValueError, match="QAT"):
        install_refiner(stub_model("B", qat=False))
    with pytest.raises(NotImplementedError, match="one residual block"):
        install_refiner(stub_model("B", blocks=2))


def test_teacher_refiner_calls_the_models_own_method():
    """The loop's distillation-teacher call (another refiner, v3.py:558-563) is not the plan's: it reaches the
    model's own _refine_logz."""
    from promptmoge_b200.integrate import install_refiner
    m = stub_model("B")
    install_refiner(m)
    with pytest.raises(AssertionError, match="not installed"):
        m._refine_logz(torch.zeros(1, 240, 320, 3), None, refiner=torch.nn.Identity())
