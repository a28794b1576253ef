"""``import turbol`` resolves to this framework (the reference's package name)."""
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_import_turbol_is_this_framework():
    code = (
        "import turbol, turbol_b200\n"
        "assert turbol is turbol_b200\n"
        "from turbol import turbol_core\n"
        "assert turbol_core is turbol_b200.turbol_core\n"
        "import turbol.vllm_inference as v\n"
        "import turbol_b200.vllm_inference as w\n"
        "assert v is w\n"
        "from turbol.rl.ppo import PPOTrainer\n"
        "from turbol_b200.rl.ppo import PPOTrainer as P2\n"
        "assert PPOTrainer is P2\n"
        "assert turbol.Tensor is turbol_core.Tensor and turbol.GPUEnvironment is turbol_core.GPUEnvironment\n"
        "assert int(turbol.StatusCode.kUnimplemented) == 5\n"
        "print('ok')\n"
    )
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr
