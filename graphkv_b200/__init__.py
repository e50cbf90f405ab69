"""graphkv_b200 -- B200-native GraphKV KV-cache compression."""
