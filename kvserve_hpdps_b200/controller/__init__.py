"""Service-aware profile selection: analytical cost model + epsilon-greedy
bandit over a profile library (reference:
kvserve_v1/compression/controller/*)."""

from kvserve_hpdps_b200.controller.analytical_model import AnalyticalModel
from kvserve_hpdps_b200.controller.bandit_state import BanditStateManager
from kvserve_hpdps_b200.controller.online_controller import OnlineController
from kvserve_hpdps_b200.controller.profile import Profile
from kvserve_hpdps_b200.controller.profile_library import ProfileLibrary

__all__ = ["AnalyticalModel", "BanditStateManager", "OnlineController", "Profile",
           "ProfileLibrary"]
