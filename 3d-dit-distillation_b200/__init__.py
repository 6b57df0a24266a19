"""vdit: B200-native sparse-voxel DiT forward path."""
