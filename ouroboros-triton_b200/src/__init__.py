"""B200-native paged block attention (drop-in for the reference `src` package)."""
