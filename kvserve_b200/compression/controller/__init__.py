"""Service-aware profile selection (behaviour of
kvserve_v1/compression/controller/*): a profile library organised by
accuracy bucket and bandwidth interval (in 1/B space), an analytical latency
model with the Theorem-1 benefit test, and an epsilon-greedy bandit that
learns the model's residuals online."""
from .profile import Profile
from .library import ProfileLibrary
from .analytical import AnalyticalModel
from .bandit import BanditStateManager
from .online import OnlineController

__all__ = ["Profile", "ProfileLibrary", "AnalyticalModel", "BanditStateManager", "OnlineController"]
