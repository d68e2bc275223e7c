"""kiwi_b200.parallel"""
