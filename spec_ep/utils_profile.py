"""The reference's import path for its profiling helpers (src/utils_profile.py, which it
installs as ``spec_ep.utils_profile``): the same names, implemented in
:mod:`spec_ep.utils.profile`, so ``from spec_ep.utils_profile import ...`` keeps working."""
from .utils.profile import (add_expert_statistics_hook, count_params, end_flops_profile, report_peak_mem,
                            save_torch_profile, start_flops_profile, torch_profile_ctx)

__all__ = ["add_expert_statistics_hook", "count_params", "end_flops_profile", "report_peak_mem",
           "save_torch_profile", "start_flops_profile", "torch_profile_ctx"]
