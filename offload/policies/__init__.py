from appcorr_b200.policies import *  # noqa: F401,F403
from appcorr_b200.policies import (SCHEDULER_REGISTRY, TRANSMISSION_REGISTRY, get_scheduler,  # noqa: F401
                                   get_transmission)
