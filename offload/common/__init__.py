from appcorr_b200.common import *  # noqa: F401,F403
from appcorr_b200.common import protocol, network, config_overrides  # noqa: F401
