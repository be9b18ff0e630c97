"""B200-native (sm_100a) per-token decoder elementwise path for NanoInfer."""
