"""B200-native decode-sampling path for Mapperatorinator-style event decoders."""
