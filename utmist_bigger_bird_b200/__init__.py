"""B200-native (sm_100a) Bigger Bird v3 sparse prefill attention."""
