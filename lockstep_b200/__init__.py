"""lockstep_b200 -- B200-native (sm_100a) LSSA-B8 / B9.1 contract attention."""
