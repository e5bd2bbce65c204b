"""B200-native FNO spectral block (drop-in for neuralop's SpectralConv inside FNOBlocks)."""
