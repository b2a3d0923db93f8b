"""B200-native sparse shared-KV attention (sm_100a)."""
