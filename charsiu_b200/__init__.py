"""charsiu-b200: a B200-native quantised-matmul device layer for charsiu."""
