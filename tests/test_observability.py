"""Env-gated diagnostics (CPU): LVSA_STEP_TIME_LOG / LVSA_MEM_LOG print at
step boundaries of both step counters, as the reference plugin does
(lvsa-vllm-omni/lvsa_vllm_omni/attention_impl.py:105-128); nothing prints
when unset; NVTX ranges are a no-op context without LVSA_NVTX."""

import contextlib

from longvideosparseattention_b200.observability import StepLogger, nvtx_range


def test_step_time_log_prints_completed_step(monkeypatch, capsys):
    monkeypatch.setenv("LVSA_STEP_TIME_LOG", "1")
    lg = StepLogger()
    lg.step_boundary(1)
    lg.step_boundary(2)
    out = capsys.readouterr().out
    assert "[LVSA-TIME] step=1 dt=" in out and "step=0" not in out


def test_logs_silent_by_default(monkeypatch, capsys):
    monkeypatch.delenv("LVSA_STEP_TIME_LOG", raising=False)
    monkeypatch.delenv("LVSA_MEM_LOG", raising=False)
    lg = StepLogger()
    lg.step_boundary(1)
    lg.step_boundary(2)
    assert capsys.readouterr().out == ""
    assert isinstance(nvtx_range("x"), contextlib.nullcontext)


def test_hook_state_logs_at_step_boundaries(monkeypatch, capsys):
    from longvideosparseattention_b200.vllm_omni.config import LVSAConfig
    from longvideosparseattention_b200.vllm_omni.hunyuan_hook import HunyuanLVSAState
    monkeypatch.setenv("LVSA_STEP_TIME_LOG", "1")
    monkeypatch.setenv("LVSA_CFG_PASSES", "1")
    s = HunyuanLVSAState(LVSAConfig())
    for _ in range(4):                  # 4 steps of 3 blocks
        for lid in (1, 2, 3):
            s.tick(lid, 100)
    lines = [l for l in capsys.readouterr().out.splitlines() if l.startswith("[LVSA-TIME]")]
    assert [l.split()[1] for l in lines] == ["step=1", "step=2"]


def test_block_count_tracker_logs(monkeypatch, capsys):
    from longvideosparseattention_b200.vllm_omni import step_tracker
    monkeypatch.setenv("LVSA_STEP_TIME_LOG", "1")
    step_tracker._logger.reset()
    t = step_tracker.BlockCountStepTracker()
    t.set_n_blocks(2)
    for _ in range(6):
        t.tick()
    lines = [l for l in capsys.readouterr().out.splitlines() if l.startswith("[LVSA-TIME]")]
    assert [l.split()[1] for l in lines] == ["step=1", "step=2"]
