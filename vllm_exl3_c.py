"""Top-level import name of the native extension the vllm-exl3 plugin loads
with ``importlib.import_module("vllm_exl3_c")`` (its NATIVE_SO hook).  It
re-exports the B200 implementation in dsv4_carve_b200.vllm_exl3_c."""
from dsv4_carve_b200.vllm_exl3_c import *  # noqa: F401,F403
from dsv4_carve_b200.vllm_exl3_c import __all__  # noqa: F401
