"""kiwi_b200.models"""
