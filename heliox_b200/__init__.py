"""heliox_b200: B200-native (sm_100a, fp64) forward + exact-adjoint path for compartmental cells."""
