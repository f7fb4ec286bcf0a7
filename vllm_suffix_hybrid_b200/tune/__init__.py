"""Online, idle-time fine-tuning of the draft head (SUFFIX_MTP_TUNE=1): see mtp_tune.py."""
